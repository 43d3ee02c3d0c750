// Query packing: builds the decode kernels' Q operand
//   qpack[g * 128 + r] = q_scale * [ q_abs(b, h) (d_c) | q_rope(b, h) (d_R) ]   (element type T)
// where q_scale = softmax_scale * log2(e), so scores come out in log2 units.
// q_abs is either given (the reference ops take it precomputed, src/fused_mla.cuh:18)
// or absorbed here: q_abs[b,h,c] = sum_i q_nope[b,h,i] * W_UK[h*dn + i, c]
// (tests/test_python.py:98-99 / tests/test_correctness.cu:29-46 of the reference).
// Padding rows of a group are written as zeros.
//
// Block (0, 0) of the absorb launch -- or of the copy launch -- also writes the
// tile prefix over groups for variable-length batches.
#include "mla_internal.cuh"

namespace mla {

// Rows given as q_absorbed: one thread per element.
template <typename T>
__global__ void pack_q_copy_kernel(DecodePlan P, const float* __restrict__ q_abs,
                                   const float* __restrict__ q_rope, float q_scale,
                                   T* __restrict__ qpack, int* tile_prefix_out) {
    clear_status(P);
    if (tile_prefix_out && blockIdx.x == 0) write_tile_prefix(P, tile_prefix_out);
    const int K = P.dc + P.dR;
    const long long total = static_cast<long long>(P.G) * kGroupRows * K;
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        int k = static_cast<int>(i % K);
        long long row = i / K;
        int g = static_cast<int>(row / kGroupRows), r = static_cast<int>(row % kGroupRows);
        int orow = group_out_row(P, g, r);
        float v = 0.f;
        if (orow >= 0) {
            v = k < P.dc ? q_abs[static_cast<long long>(orow) * P.dc + k]
                         : q_rope[static_cast<long long>(orow) * P.dR + (k - P.dc)];
            v *= q_scale;
        }
        qpack[i] = ElemTraits<T>::from_f(v);
    }
}

// Absorption: block (h, chunk of kTok tokens), 256 threads. W_UK[h] is (dn, dc)
// row-major. Thread (rg, cg) owns the 8 output columns [8 cg, 8 cg + 8) and the
// rows i = rg, rg + RG, ... (RG = 256 / (dc / 8) row groups): it streams 16-byte
// vectors of W_UK, so the block keeps 256 independent loads in flight and reads
// W_UK[h] exactly once per token chunk. Row-group partial sums are reduced
// through shared memory.
template <typename T, int kTok>
__global__ void __launch_bounds__(256)
pack_q_absorb_kernel(DecodePlan P, const float* __restrict__ q_nope, const T* __restrict__ W_UK,
                     const float* __restrict__ q_rope, float q_scale, T* __restrict__ qpack,
                     int* tile_prefix_out) {
    clear_status(P);
    if (tile_prefix_out && blockIdx.x == 0 && blockIdx.y == 0) write_tile_prefix(P, tile_prefix_out);
    extern __shared__ float smem[];
    const int h = blockIdx.x;
    const int b0 = blockIdx.y * kTok;
    const int dn = P.dn, dc = P.dc, K = P.dc + P.dR;
    const int ntok = (P.B - b0) < kTok ? (P.B - b0) : kTok;
    float* qn_s = smem;                    // kTok * dn
    float* red = smem + kTok * dn;         // RG * kTok * dc partial sums
    for (int i = threadIdx.x; i < kTok * dn; i += blockDim.x) {
        int t = i / dn, d = i % dn;
        qn_s[i] = t < ntok ? q_nope[(static_cast<long long>(b0 + t) * P.H + h) * dn + d] : 0.f;
    }
    __syncthreads();
    const int ncg = dc / 8;                       // column groups (dc is a multiple of 32)
    const int RG = blockDim.x / ncg > 0 ? blockDim.x / ncg : 1;
    const T* W = W_UK + static_cast<long long>(h) * dn * dc;
    for (int cg0 = 0; cg0 < ncg; cg0 += blockDim.x / RG) {
        const int cg = cg0 + static_cast<int>(threadIdx.x) % (blockDim.x / RG);
        const int rg = static_cast<int>(threadIdx.x) / (blockDim.x / RG);
        float acc[kTok][8];
#pragma unroll
        for (int t = 0; t < kTok; ++t)
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[t][e] = 0.f;
        if (cg < ncg && rg < RG) {
#pragma unroll 4
            for (int i = rg; i < dn; i += RG) {
                const uint4 v = __ldg(reinterpret_cast<const uint4*>(W + static_cast<long long>(i) * dc + 8 * cg));
                const uint32_t* u = reinterpret_cast<const uint32_t*>(&v);
                float w[8];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 f = ElemTraits<T>::to_f2(*reinterpret_cast<const typename ElemTraits<T>::T2*>(&u[e]));
                    w[2 * e] = f.x;
                    w[2 * e + 1] = f.y;
                }
#pragma unroll
                for (int t = 0; t < kTok; ++t) {
                    const float q = qn_s[t * dn + i];
#pragma unroll
                    for (int e = 0; e < 8; ++e) acc[t][e] = fmaf(q, w[e], acc[t][e]);
                }
            }
            for (int t = 0; t < ntok; ++t)
#pragma unroll
                for (int e = 0; e < 8; ++e) red[(rg * kTok + t) * dc + 8 * cg + e] = acc[t][e];
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < ntok * dc; i += blockDim.x) {
        const int t = i / dc, c = i % dc;
        float a = 0.f;
        for (int rg = 0; rg < RG; ++rg) a += red[(rg * kTok + t) * dc + c];
        const int b = b0 + t;
        const long long qrow = P.shared ? static_cast<long long>(b) * P.H + h
                                        : static_cast<long long>(b) * P.head_blocks * kGroupRows + h;
        qpack[qrow * K + c] = ElemTraits<T>::from_f(a * q_scale);
    }
    // rope part
    for (int i = threadIdx.x; i < ntok * P.dR; i += blockDim.x) {
        const int t = i / P.dR, j = i % P.dR;
        const int b = b0 + t;
        const int flat = b * P.H + h;
        const long long qrow = P.shared ? flat : static_cast<long long>(b) * P.head_blocks * kGroupRows + h;
        qpack[qrow * K + P.dc + j] =
            ElemTraits<T>::from_f(q_rope[static_cast<long long>(flat) * P.dR + j] * q_scale);
    }
}

// Zero the padding rows of every group (rows whose output row is -1).
template <typename T>
__global__ void pack_q_zero_pad_kernel(DecodePlan P, T* __restrict__ qpack) {
    const int K = P.dc + P.dR;
    const long long total = static_cast<long long>(P.G) * kGroupRows * K;
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        long long row = i / K;
        int g = static_cast<int>(row / kGroupRows), r = static_cast<int>(row % kGroupRows);
        if (group_out_row(P, g, r) < 0) qpack[i] = ElemTraits<T>::from_f(0.f);
    }
}

template <typename T>
cudaError_t launch_pack_q(const DecodePlan& P, const float* q_absorbed, const float* q_nope,
                          const T* W_UK, const float* q_rope, float q_scale, T* qpack,
                          int* tile_prefix_out, cudaStream_t s) {
    const long long total = static_cast<long long>(P.G) * kGroupRows * (P.dc + P.dR);
    int blocks = static_cast<int>((total + 255) / 256);
    if (blocks > 4096) blocks = 4096;
    if (q_absorbed) {
        pack_q_copy_kernel<T><<<blocks, 256, 0, s>>>(P, q_absorbed, q_rope, q_scale, qpack,
                                                     tile_prefix_out);
        count_launches(1);
        return cudaGetLastError();
    }
    bool has_pad = P.shared ? (P.B * P.H) % kGroupRows != 0 : P.H % kGroupRows != 0;
    if (has_pad) {
        pack_q_zero_pad_kernel<T><<<blocks, 256, 0, s>>>(P, qpack);
        count_launches(1);
    }
    constexpr int kTok = 4;
    dim3 grid(P.H, ceil_div(P.B, kTok));
    const int ncg = P.dc / 8;
    const int RG = 256 / ncg > 0 ? 256 / ncg : 1;
    size_t smem = (static_cast<size_t>(kTok) * P.dn + static_cast<size_t>(RG) * kTok * P.dc) * sizeof(float);
    if (smem > 48 * 1024) {
        cudaError_t e =
            ensure_dynamic_smem(reinterpret_cast<const void*>(pack_q_absorb_kernel<T, kTok>), static_cast<int>(smem));
        if (e != cudaSuccess) return e;
    }
    pack_q_absorb_kernel<T, kTok><<<grid, 256, smem, s>>>(P, q_nope, W_UK, q_rope, q_scale, qpack,
                                                          tile_prefix_out);
    count_launches(1);
    return cudaGetLastError();
}

template <typename T>
cudaError_t launch_pack_zero_pad(const DecodePlan& P, T* qpack, cudaStream_t s) {
    const bool has_pad = P.shared ? (P.B * P.H) % kGroupRows != 0 : P.H % kGroupRows != 0;
    if (!has_pad) return cudaSuccess;
    const long long total = static_cast<long long>(P.G) * kGroupRows * (P.dc + P.dR);
    int blocks = static_cast<int>((total + 255) / 256);
    if (blocks > 4096) blocks = 4096;
    pack_q_zero_pad_kernel<T><<<blocks, 256, 0, s>>>(P, qpack);
    count_launches(1);
    return cudaGetLastError();
}

template cudaError_t launch_pack_zero_pad<__half>(const DecodePlan&, __half*, cudaStream_t);
template cudaError_t launch_pack_zero_pad<__nv_bfloat16>(const DecodePlan&, __nv_bfloat16*, cudaStream_t);
template cudaError_t launch_pack_q<__half>(const DecodePlan&, const float*, const float*, const __half*,
                                           const float*, float, __half*, int*, cudaStream_t);
template cudaError_t launch_pack_q<__nv_bfloat16>(const DecodePlan&, const float*, const float*,
                                                  const __nv_bfloat16*, const float*, float,
                                                  __nv_bfloat16*, int*, cudaStream_t);

}  // namespace mla
