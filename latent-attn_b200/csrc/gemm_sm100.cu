// Tensor-core (tcgen05) GEMMs on either side of the decode kernel.
//
// 1. Query absorption, per head h:
//        q_abs[b, h, :] = q_nope[b, h, :] . W_UK[h*dn : (h+1)*dn, :]      (dn x d_c)
//    (the absorption of tests/test_python.py:98-99 / tests/test_correctness.cu:29-46
//    in the reference, done there on the caller side) written straight into the
//    decode kernel's packed query rows qpack = q_scale * [q_abs | q_rope].
//    It runs transposed, D^T[d_c x tokens] = W_UK_h^T . q_nope_h^T, so the 128-row
//    M tile is a slice of d_c and any token count (1 .. 256 per CTA) is the N side:
//      A = W_UK_h^T, MN-major (d_c contiguous), 2 TMA boxes of 64 d_c x dn rows
//      B = q_nope_h^T, K-major, converted from fp32 on load into two 16-bit parts, hi =
//          round(q) and lo = round(q - hi), and both are multiplied (two K passes into one
//          accumulator): the product keeps q_nope to about 2^-17 instead of the 2^-9 of a
//          single bf16 rounding, the largest error term of the whole decode for short sequences.
//    CTA = (d_c slice of 128, head, block of up to 128 tokens), 128 threads.
//
// 2. Split-KV merge + output projection, per head h:
//        o_lat[b, h, :] = sum_k w_k o_k     (log-sum-exp weights of the partial records)
//        out[b, h, j]   = o_lat[b, h, :] . W_UV[h*dv + j, :]   (src/fused_mla.cu:258-267)
//    Transposed again, D^T[dv x tokens] = W_UV_h . o_lat_h^T with M = dv = 128:
//      A = W_UV_h, K-major, all d_c / 64 TMA boxes resident (128 KB at d_c = 512)
//      B = o_lat_h^T, K-major, merged by the CTA's threads from the records (L2) in one pass:
//          each record's (m, l) is loaded with its row and folded into a running log-sum-exp.
//    CTA = (block of up to 64 tokens, head), 512 threads. The same kernel merges the gathered
//    partial sets of KV-range shards (mla_combine_partials).
//
// Batches of at most four tokens take fp32 CUDA-core kernels instead (absorb_gemv_kernel,
// project_gemv_kernel): there both products are matrix-vector products bound by reading the
// weights once, and fp32 operands need no hi/lo split.
//
// The projection kernels launch their W loads by TMA before waiting on the previous kernel
// (programmatic dependent launch), so weight streaming overlaps its tail.
// Every wait is bounded; on timeout the status word records it.
#include <algorithm>
#include <cfloat>
#include <cstdlib>

#include "mla_internal.cuh"
#include "sm100_ptx.cuh"
#include "tma_host.cuh"
#include "proj_unit.cuh"
#include "peer.cuh"

namespace mla {
using namespace sm100;

namespace {

template <typename T> struct GemmFmt;
template <> struct GemmFmt<__half> { static constexpr uint32_t v = 0; };
template <> struct GemmFmt<__nv_bfloat16> { static constexpr uint32_t v = 1; };

template <typename T>
__device__ __forceinline__ uint32_t pack_pair(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack_pair<__half>(float a, float b) {
    __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
}
template <>
__device__ __forceinline__ uint32_t pack_pair<__nv_bfloat16>(float a, float b) {
    __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}
// query-pack row of token n (single query per sequence: n = b; shared cache: flattened)
__device__ __forceinline__ long long qpack_row(const DecodePlan& P, int b, int h) {
    return P.shared ? static_cast<long long>(b) * P.H + h
                    : static_cast<long long>(b) * P.head_blocks * kGroupRows + h;
}

constexpr int kAbsorbTok = 128;    // tokens per absorption CTA (MMA M)
constexpr int kAbsorbThreads = 256;
using proj::kProjTok;               // tokens per projection CTA
constexpr int kProjWarps = 16;     // projection CTA: 16 warps merge, warp 0 issues the MMA, warps 4-7 store

// absorption shared memory: W_UK_h (d_c / 64 boxes of dn rows x 128 B), the hi and lo A parts, barriers
__host__ __device__ inline size_t absorb_smem_bytes(int dn, int dc) {
    return static_cast<size_t>(dc / 64) * dn * 128 + 2 * static_cast<size_t>(dn / 64) * kAbsorbTok * 128 + 32;
}

constexpr float kLn2 = 0.6931471805599453f;

enum : int { kSiteAbsorbA = 12, kSiteAbsorbMma = 13, kSiteProjA = 14, kSiteProjMma = 15 };
__device__ __forceinline__ int gcode(int site) { return kStatusTimeout | (site << 8); }

}  // namespace

// ------------------------------------------------------------------------------------------
// absorption
// ------------------------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(kAbsorbThreads, 1)
absorb_sm100_kernel(const __grid_constant__ CUtensorMap tmap_w, const DecodePlan P, const float* __restrict__ q_nope,
                    const float* __restrict__ q_rope, float q_scale, T* __restrict__ qpack, int* tile_prefix_out) {
    // CTA = (block of up to 128 tokens, head h), 256 threads. D[tokens x d_c] = q_nope_h . W_UK_h in TMEM
    // (lane = token, column = d_c index), in N = 256 column halves:
    //   A = q_nope_h rows, K-major (K = dn), 128-byte swizzle, hi and lo parts (dn / 64 chunks each)
    //   B = W_UK_h, MN-major (d_c contiguous): d_c / 64 TMA boxes of 64 columns x dn rows
    clear_status(P);
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const int dn = P.dn, dc = P.dc, dR = P.dR, K = P.dc + P.dR;   // dn == 128, dc % 256 == 0, dc <= 512
    const int box_bytes = dn * 128;                                // one W box: 64 d_c x dn rows
    const int nbox = dc / 64;
    const uint32_t w_u32 = smem_u32(smem);
    const uint32_t a_u32 = w_u32 + nbox * box_bytes;               // [part][dn / 64][128 rows x 128 B]
    const uint32_t chunk_bytes = kAbsorbTok * 128;
    const uint32_t part_bytes = (dn / 64) * chunk_bytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + nbox * box_bytes + 2 * part_bytes);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2);
    const uint32_t w_full = smem_u32(&bars[0]), mma_done = smem_u32(&bars[1]);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int b0 = blockIdx.x * kAbsorbTok, h = blockIdx.y;
    const int ntok = min(kAbsorbTok, P.B - b0);
    volatile int* err = P.status;

    pdl_launch_dependents();
    if (tile_prefix_out && blockIdx.x == 0 && blockIdx.y == 0) write_tile_prefix(P, tile_prefix_out);
    if (threadIdx.x == 0) {
        mbar_init(w_full, 1);
        mbar_init(mma_done, 1);
        fence_mbar_init();
        tma_prefetch_desc(&tmap_w);
        mbar_arrive_expect_tx(w_full, static_cast<uint32_t>(nbox * box_bytes));
        for (int j = 0; j < nbox; ++j) tma_load_2d(w_u32 + j * box_bytes, &tmap_w, w_full, 64 * j, h * dn);
    }
    if (warp == 0) {
        tmem_alloc(smem_u32(tmem_slot), 512);
        tmem_relinquish();
    }
    // Thread (t, half): token t's q_nope elements [64 half, 64 half + 64) (A chunk `half`) and rope
    // elements [dR/2 half, dR/2 (half + 1)); every load is issued before the first is used.
    const int t = threadIdx.x & (kAbsorbTok - 1), half = threadIdx.x / kAbsorbTok;
    const bool tok = t < ntok;
    const long long flat = static_cast<long long>(b0 + t) * P.H + h;
    float4 x[16];
    float4 r[8];
    const int rq = dR / 8;   // float4 units of a rope half (dR % 8 == 0, dR <= 64)
#pragma unroll
    for (int u = 0; u < 16; ++u)
        x[u] = tok ? __ldg(reinterpret_cast<const float4*>(q_nope + flat * dn + 64 * half) + u)
                   : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int u = 0; u < 8; ++u)
        r[u] = (tok && u < rq) ? __ldg(reinterpret_cast<const float4*>(q_rope + flat * dR + (dR / 2) * half) + u)
                               : make_float4(0.f, 0.f, 0.f, 0.f);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tmem_slot;
    {
        // hi = round(q), lo = round(q - hi): 16-byte units u of row t, swizzled by (t % 8)
        const uint32_t row = a_u32 + half * chunk_bytes + t * 128;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const float v[8] = {x[2 * u].x, x[2 * u].y, x[2 * u].z, x[2 * u].w,
                                x[2 * u + 1].x, x[2 * u + 1].y, x[2 * u + 1].z, x[2 * u + 1].w};
            uint32_t hi[4], lo[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                hi[e] = pack_pair<T>(v[2 * e], v[2 * e + 1]);
                const float2 hv = ElemTraits<T>::to_f2(*reinterpret_cast<const typename ElemTraits<T>::T2*>(&hi[e]));
                lo[e] = pack_pair<T>(v[2 * e] - hv.x, v[2 * e + 1] - hv.y);
            }
            const uint32_t dst = row + ((u ^ (t & 7)) << 4);
            st_shared_v4(dst, hi[0], hi[1], hi[2], hi[3]);
            st_shared_v4(dst + part_bytes, lo[0], lo[1], lo[2], lo[3]);
        }
        // rope columns: scaled and rounded once, written straight to qpack
        if (tok) {
            T* dst = qpack + qpack_row(P, b0 + t, h) * K + dc + (dR / 2) * half;
#pragma unroll
            for (int u = 0; u < 8; u += 2) {
                if (u < rq) {
                    const uint4 y = make_uint4(pack_pair<T>(r[u].x * q_scale, r[u].y * q_scale),
                                               pack_pair<T>(r[u].z * q_scale, r[u].w * q_scale),
                                               pack_pair<T>(r[u + 1].x * q_scale, r[u + 1].y * q_scale),
                                               pack_pair<T>(r[u + 1].z * q_scale, r[u + 1].w * q_scale));
                    *reinterpret_cast<uint4*>(dst + 4 * u) = y;
                }
            }
        }
    }
    fence_proxy_async_smem();
    __syncthreads();
    bool issued = true;   // thread 0: W_UK landed and the MMAs were issued
    if (threadIdx.x == 0) {
        // a wait that ends only on completion or its time limit: shared memory must not be released
        // under a TMA write
        issued = mbar_wait_impl<false, false>(w_full, 0, err, gcode(kSiteAbsorbA), kDefaultWaitNs);
        if (issued) {
            tc_fence_after();
            const uint32_t idesc = idesc_f16(128, 256, GemmFmt<T>::v, false, true);
            for (int nh = 0; nh < dc / 256; ++nh)
                for (int part = 0; part < 2; ++part)   // hi, then lo, into the same accumulator
                    for (int k = 0; k < dn / 16; ++k) {
                        const uint64_t ad = smem_desc_sw128(a_u32 + part * part_bytes + (k >> 2) * chunk_bytes +
                                                                (k & 3) * 32, 16, 1024);
                        const uint64_t bd = smem_desc_sw128(w_u32 + nh * 4 * box_bytes + k * 2048, box_bytes, 1024);
                        mma_ss(tbase + nh * 256, ad, bd, idesc, (part | k) > 0 ? 1u : 0u);
                    }
        }
        mma_commit(mma_done);  // also arrives when nothing was issued
    }
    // epilogue: warp w reads TMEM lanes 32 (w % 4) .. + 31 (its tokens) and the d_c columns of half
    // w / 4, scales and rounds them into token rows of T in shared memory (the W_UK space, free once
    // the MMAs completed; 16-byte units swizzled by token % 8), and the block then writes the rows to
    // qpack with coalesced 16-byte stores (a warp covers 512 contiguous bytes).
    bool ok = mbar_wait(mma_done, 0, err, gcode(kSiteAbsorbMma));
    ok = __syncthreads_and(ok && (threadIdx.x != 0 || issued));
    if (ok) {
        tc_fence_after();
        const int tt = 32 * (warp & 3) + lane, ch = warp >> 2;
        const uint32_t trow = tbase + (static_cast<uint32_t>(32 * (warp & 3)) << 16);
        const uint32_t srow = w_u32 + tt * (dc * 2);
        for (int c0 = ch * (dc / 2); c0 < (ch + 1) * (dc / 2); c0 += 32) {
            uint32_t v[32];
            tmem_ld32_sync(trow + c0, v);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int j = c0 / 8 + q;   // 16-byte unit of the row
                st_shared_v4(srow + (((j & ~7) | ((j & 7) ^ (tt & 7))) << 4),
                             pack_pair<T>(__uint_as_float(v[8 * q + 0]) * q_scale, __uint_as_float(v[8 * q + 1]) * q_scale),
                             pack_pair<T>(__uint_as_float(v[8 * q + 2]) * q_scale, __uint_as_float(v[8 * q + 3]) * q_scale),
                             pack_pair<T>(__uint_as_float(v[8 * q + 4]) * q_scale, __uint_as_float(v[8 * q + 5]) * q_scale),
                             pack_pair<T>(__uint_as_float(v[8 * q + 6]) * q_scale, __uint_as_float(v[8 * q + 7]) * q_scale));
            }
        }
        __syncthreads();
        const int upr = dc / 8;   // 16-byte units per row
        for (int i2 = threadIdx.x; i2 < ntok * upr; i2 += blockDim.x) {
            const int tk = i2 / upr, j = i2 % upr;
            const uint4 y = *reinterpret_cast<const uint4*>(smem + tk * (dc * 2) + ((((j & ~7) | ((j & 7) ^ (tk & 7)))) << 4));
            *reinterpret_cast<uint4*>(qpack + qpack_row(P, b0 + tk, h) * K + 8 * j) = y;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tbase, 512);
    }
    // a W_UK wait that gave up: wait (bounded) for the boxes before the shared memory is released
    if (threadIdx.x == 0 && !issued) mbar_wait_impl<false, false>(w_full, 0, err, gcode(kSiteAbsorbA), 100000000ull);
}

// ------------------------------------------------------------------------------------------
// absorption of a few tokens: fp32 CUDA-core GEMV
// ------------------------------------------------------------------------------------------
// For B <= kAbsorbGemvTok the absorption is a vector-matrix product per token and head (dn x d_c),
// bound by reading W_UK once. The products are formed in fp32 from the fp32 q_nope (no rounding of
// the query before the product). CTA = (slice of 256 d_c columns, head h), 256 threads: warp w takes
// the W_UK rows i = 16 w .. 16 w + 15 and lane l the 8 columns 8 l .. 8 l + 7 of the slice, with all
// 16 row loads in flight at once; the 8 warps' partial sums are added in warp order through shared
// memory, scaled, rounded once to T and written as 16-byte rows of qpack.
constexpr int kAbsorbGemvTok = 4;
constexpr int kAbsorbGemvCols = 256;

template <typename T>
__global__ void __launch_bounds__(256)
absorb_gemv_kernel(const DecodePlan P, const float* __restrict__ q_nope, const T* __restrict__ W_UK,
                   const float* __restrict__ q_rope, float q_scale, T* __restrict__ qpack, int* tile_prefix_out) {
    clear_status(P);
    __shared__ float red[8][kAbsorbGemvTok][kAbsorbGemvCols];   // 32 KB
    const int dn = P.dn, dc = P.dc, K = P.dc + P.dR, B = P.B;   // dn == 128, dc % 256 == 0, B <= 4
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int c0 = blockIdx.x * kAbsorbGemvCols, h = blockIdx.y;
    pdl_launch_dependents();
    if (tile_prefix_out && blockIdx.x == 0 && blockIdx.y == 0) write_tile_prefix(P, tile_prefix_out);
    using T2 = typename ElemTraits<T>::T2;
    {
        uint4 wv[16];
        const T* wrow = W_UK + (static_cast<long long>(h) * dn + 16 * warp) * dc + c0 + 8 * lane;
#pragma unroll
        for (int i = 0; i < 16; ++i) wv[i] = __ldg(reinterpret_cast<const uint4*>(wrow + static_cast<long long>(i) * dc));
        float acc[kAbsorbGemvTok][8];
#pragma unroll
        for (int t = 0; t < kAbsorbGemvTok; ++t)
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[t][e] = 0.f;
#pragma unroll
        for (int t = 0; t < kAbsorbGemvTok; ++t) {
            if (t < B) {
                // lanes 0-15 hold this warp's 16 q_nope values of token t; broadcast by shuffle
                const float qv = lane < 16 ? __ldg(q_nope + (static_cast<long long>(t) * P.H + h) * dn + 16 * warp + lane)
                                           : 0.f;
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const float q = __shfl_sync(0xffffffffu, qv, i);
                    const float2 a = ElemTraits<T>::to_f2(*reinterpret_cast<const T2*>(&wv[i].x));
                    const float2 b = ElemTraits<T>::to_f2(*reinterpret_cast<const T2*>(&wv[i].y));
                    const float2 c = ElemTraits<T>::to_f2(*reinterpret_cast<const T2*>(&wv[i].z));
                    const float2 d = ElemTraits<T>::to_f2(*reinterpret_cast<const T2*>(&wv[i].w));
                    acc[t][0] = fmaf(q, a.x, acc[t][0]); acc[t][1] = fmaf(q, a.y, acc[t][1]);
                    acc[t][2] = fmaf(q, b.x, acc[t][2]); acc[t][3] = fmaf(q, b.y, acc[t][3]);
                    acc[t][4] = fmaf(q, c.x, acc[t][4]); acc[t][5] = fmaf(q, c.y, acc[t][5]);
                    acc[t][6] = fmaf(q, d.x, acc[t][6]); acc[t][7] = fmaf(q, d.y, acc[t][7]);
                }
                float4* dst = reinterpret_cast<float4*>(&red[warp][t][8 * lane]);
                dst[0] = make_float4(acc[t][0], acc[t][1], acc[t][2], acc[t][3]);
                dst[1] = make_float4(acc[t][4], acc[t][5], acc[t][6], acc[t][7]);
            }
        }
    }
    __syncthreads();
    // (token, 8-column group) items: sum the 8 warps in order, scale, round, one 16-byte store
    for (int i = threadIdx.x; i < B * (kAbsorbGemvCols / 8); i += blockDim.x) {
        const int t = i / (kAbsorbGemvCols / 8), g = i % (kAbsorbGemvCols / 8);
        float v[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            float s = 0.f;
#pragma unroll
            for (int w = 0; w < 8; ++w) s += red[w][t][8 * g + e];
            v[e] = s * q_scale;
        }
        const uint4 x = make_uint4(pack_pair<T>(v[0], v[1]), pack_pair<T>(v[2], v[3]), pack_pair<T>(v[4], v[5]),
                                   pack_pair<T>(v[6], v[7]));
        *reinterpret_cast<uint4*>(qpack + qpack_row(P, t, h) * K + c0 + 8 * g) = x;
    }
    if (blockIdx.x == 0) {
        // rope columns, 4 at a time
        const int q4 = P.dR / 4;
        for (int i = threadIdx.x; i < B * q4; i += blockDim.x) {
            const int t = i / q4, j = 4 * (i % q4);
            const long long flat = static_cast<long long>(t) * P.H + h;
            const float4 x = *reinterpret_cast<const float4*>(q_rope + flat * P.dR + j);
            const uint2 y = make_uint2(pack_pair<T>(x.x * q_scale, x.y * q_scale), pack_pair<T>(x.z * q_scale, x.w * q_scale));
            *reinterpret_cast<uint2*>(qpack + qpack_row(P, t, h) * K + dc + j) = y;
        }
    }
}

// ------------------------------------------------------------------------------------------
// merge + projection
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}
__device__ __forceinline__ void prefetch_l2(const void* p) {
    asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

// One CTA per (block of up to 64 tokens, head); the unit's steps are in proj_unit.cuh.
template <typename T, typename R>
__global__ void __launch_bounds__(32 * kProjWarps)
project_sm100_kernel(const __grid_constant__ CUtensorMap tmap_w, const DecodePlan P, const float* __restrict__ rec_ml,
                     const R* __restrict__ rec_o, float* __restrict__ out, int ntp, uint32_t tmem_cols,
                     int parts, int ml_stride, int o_stride, int prefetch_stride) {
    // parts == 0 (R = T): the decode kernel's partial records (m in log2 units, o rounded to T, or
    // o / l for fp16, record g + w of group g). parts > 0 (R = float): that many partial sets of [part][B][H] rows
    // (m, l at rec_ml + row * ml_stride, unnormalised o at rec_o + row * o_stride: the separate arrays
    // of mla_decode_partial or its packed rows), with m in natural-log units and l = 0 for an empty
    // part (the KV-range shards' merge).
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const int dc = P.dc, dv = P.dv;
    const int nk = dc / 64;                                   // K chunks
    const uint32_t a_u32 = smem_u32(smem);                    // nk x (dv rows x 128 B)
    const uint32_t b_u32 = a_u32 + nk * dv * 128;             // nk x (ntp rows x 128 B)
    unsigned char* tail = smem + nk * dv * 128 + nk * ntp * 128;
    proj::Lists* L = reinterpret_cast<proj::Lists*>(tail);
    float* red = reinterpret_cast<float*>(tail + sizeof(proj::Lists));   // split partial sums: red_rows(ntp) x d_c
    uint64_t* bars = reinterpret_cast<uint64_t*>(tail + sizeof(proj::Lists) +
                                                 static_cast<size_t>(proj::red_rows(ntp)) * dc * sizeof(float));
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2);
    const uint32_t a_full = smem_u32(&bars[0]), mma_done = smem_u32(&bars[1]);

    const int warp = threadIdx.x >> 5;
    const int b0 = blockIdx.x * kProjTok, h = blockIdx.y;
    const int ntok = min(kProjTok, P.B - b0);
    volatile int* err = P.status;

    if (threadIdx.x == 0) {
        mbar_init(a_full, 1);
        mbar_init(mma_done, 1);
        fence_mbar_init();
        tma_prefetch_desc(&tmap_w);
    }
    if (warp == 0) {
        tmem_alloc(smem_u32(tmem_slot), tmem_cols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tmem_slot;
    if (threadIdx.x == 0) {
        // W_UV rows of head h do not depend on the decode kernel: stream them now
        mbar_arrive_expect_tx(a_full, static_cast<uint32_t>(nk * dv * 128));
        for (int j = 0; j < nk; ++j) tma_load_2d(a_u32 + j * dv * 128, &tmap_w, a_full, 64 * j, h * dv);
    }
    // With uniform lengths (or partial sets) the record lists are arithmetic on the plan and are
    // built before the wait on the decode kernel; with variable lengths they read the tile prefix,
    // which is complete only when that wait returns.
    const bool lists_early = parts > 0 || P.uniform_len > 0;
    if (!lists_early) pdl_wait();
    const int step = parts ? P.B * P.H : kGroupRows;          // rows between a token's consecutive records
    const int ntiles = parts ? 0 : total_tiles(P);
    proj::build_lists(P, L, b0, ntok, h, parts, ntiles);
    __syncthreads();
    if (lists_early) pdl_wait();  // records and status come from the decode kernel
    // The status load is issued now and consumed after the merge, so it overlaps the record loads;
    // a failed decode leaves garbage in the records, which are merged but never multiplied.
    const int status0 = *err;
    // With more CTAs than SMs, the CTA `prefetch_stride` positions later in launch order runs on an
    // SM after one of this wave: its records are prefetched into L2 now, so its merge reads L2.
    {
        const int nxt = blockIdx.x + gridDim.x * blockIdx.y + prefetch_stride;
        if (prefetch_stride > 0 && nxt < static_cast<int>(gridDim.x * gridDim.y)) {
            const int xb = nxt % gridDim.x, hh = nxt / gridDim.x;
            const int nt = min(kProjTok, P.B - xb * kProjTok);
            for (int t = threadIdx.x; t < nt; t += blockDim.x) {
                int n, w0, base;
                proj::record_list(P, xb * kProjTok + t, hh, parts, ntiles, n, w0, base);
                for (int k = 0; k < n; ++k) {
                    const long long row = static_cast<long long>(base) + static_cast<long long>(k) * step;
                    prefetch_l2_bulk(rec_o + row * o_stride, static_cast<uint32_t>(dc * sizeof(R)));
                    prefetch_l2(rec_ml + row * ml_stride);
                }
            }
        }
    }
    proj::merge<T, R, kProjWarps>(P, L, red, b_u32, ntok, ntp, parts, ml_stride, o_stride, rec_ml, rec_o);
    const bool failed = parts == 0 && status0 != kStatusOk;
    fence_proxy_async_smem();
    __syncthreads();
    bool issued = true;   // thread 0: the W_UV boxes landed (and, unless failed, the MMAs were issued)
    if (threadIdx.x == 0) {
        // always wait for the W_UV boxes: shared memory must not be released under a TMA write
        issued = mbar_wait(a_full, 0, err, gcode(kSiteProjA));
        if (issued && !failed) {
            tc_fence_after();
            proj::issue_mma<T>(tbase, a_u32, b_u32, dc, dv, ntp);
        }
        mma_commit(mma_done);
    }
    if (warp == 0 || (warp >= 4 && warp < 8)) {
        // thread 0's result reaches the epilogue warps through an AND over a named barrier of
        // warps 0 and 4-7 (no global status read)
        issued = proj::bar_and(1, 160, issued);
    }
    if (warp >= 4 && warp < 8) {
        bool ok = mbar_wait(mma_done, 0, err, gcode(kSiteProjMma)) && issued && !failed;
        ok = __all_sync(0xffffffffu, ok);
        // a failed decode, or a wait that gave up (the status word holds where): the output shows it
        proj::store_out(P, tbase, out, b0, ntok, h, ok);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        // the MMAs (if any) completed: mma_done was waited on by warps 4-7
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tbase, tmem_cols);
    }
}

// ------------------------------------------------------------------------------------------
// launch helpers
// ------------------------------------------------------------------------------------------
namespace {
uint32_t tmem_cols_for(int n) {
    uint32_t c = 32;
    while (c < static_cast<uint32_t>(n)) c <<= 1;
    return c;
}
int pad16(int n) { return (n + 15) / 16 * 16; }

template <typename Kernel, typename... Args>
cudaError_t launch_ex(Kernel k, dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k, args...);
}
}  // namespace

// ------------------------------------------------------------------------------------------
// merge + projection of a few tokens: fp32 CUDA-core GEMV
// ------------------------------------------------------------------------------------------
// For B <= kGemvMaxTok the W_UV product is a matrix-vector product per token (128 x d_c per
// head), too small for the tensor cores to pay for their issue and TMEM round trip, and the merged
// latent row can stay in fp32 (no rounding before the projection). One CTA per head h, 512 threads:
//   0. thread 0 starts the TMA of W_UV[h] (dv x d_c, independent of the decode kernel) before the
//      programmatic-dependent wait;
//   1. warps are split over the tokens (16 / B warps each); a warp merges the records k = s, s + S, ...
//      of its token, four per round trip, into a running log-sum-exp (max, row sum, rescaled sum);
//   2. per token, the warp partials are rescaled to the common max and summed column by column into
//      the fp32 latent row (shared memory);
//   3. thread (q, j) dots W_UV row j with latent quarter q for every token (each W element read once
//      from shared memory per CTA); the four quarters are summed in a fixed order.
constexpr int kGemvWarps = 16;
constexpr int kGemvRec = 4;      // records per warp per round trip
constexpr int kGemvMaxTok = 4;   // batches up to this size take the GEMV kernel

__host__ __device__ inline size_t gemv_smem_bytes(int dc, int dv) {
    return static_cast<size_t>(dc / 64) * dv * 128 +             // W_UV[h] boxes
           static_cast<size_t>(kGemvWarps) * dc * sizeof(float) + // warp partial sums
           kGemvWarps * sizeof(float2) +                          // warp (max, row sum)
           static_cast<size_t>(kGemvMaxTok) * dc * sizeof(float) +   // merged latent rows
           static_cast<size_t>(4) * kGemvMaxTok * dv * sizeof(float) +  // quarter sums
           16;                                                    // mbarrier
}

// Step 1 of the GEMV merge, shared by the projection and the partial export: warp w takes token
// t = w / wpt and records k = s, s + wpt, ... (s = w % wpt) of head h, and leaves its running
// (max in log2 units, row sum) in wml[w] and its unnormalised latent sum at that max in red[w].
// With uniform lengths (or partial sets) the record list is arithmetic on the plan and is built
// before the wait on the previous kernel; with variable lengths it reads the tile prefix.
// Returns the decode status word as read after that wait.
template <typename R>
__device__ __forceinline__ int gemv_merge(const DecodePlan& P, const float* __restrict__ rec_ml,
                                          const R* __restrict__ rec_o, int parts, int ml_stride, int o_stride, int h,
                                          float* red, float2* wml) {
    const int dc = P.dc, B = P.B;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    volatile int* err = P.status;
    const int step = parts ? B * P.H : kGroupRows;
    const float mscale = parts ? 1.4426950408889634f : 1.f;   // m in log2 units

    const int wpt = kGemvWarps / B;
    const int t = warp / wpt, s = warp % wpt;
    const bool lists_early = parts > 0 || P.uniform_len > 0;
    if (!lists_early) pdl_wait();
    const int ntiles = parts ? 0 : total_tiles(P);
    const bool busy = parts || ntiles >= P.W;   // every worker owns a tile: every record in the range exists
    int n = 0, w0 = 0, base = 0;
    if (t < B) proj::record_list(P, t, h, parts, ntiles, n, w0, base);
    if (lists_early) pdl_wait();  // records and status come from the decode kernel
    const int status0 = *err;     // consumed after the merge
    if (t < B) {
        const float4 zero4 = make_float4(0.f, 0.f, 0.f, 0.f);
        float mrun = -INFINITY, lrun = 0.f;
        float4 acc[4] = {zero4, zero4, zero4, zero4};
        for (int k0 = s; k0 < n; k0 += wpt * kGemvRec) {
            float2 mlq[kGemvRec];
            float4 v[kGemvRec][4];
#pragma unroll
            for (int q = 0; q < kGemvRec; ++q) {
                const int k = k0 + q * wpt;
                // a worker that owns no tile of the group wrote no record: it is never read
                const bool in = k < n && (busy ||
                                          worker_begin(ntiles, P.W, w0 + k) != worker_begin(ntiles, P.W, w0 + k + 1));
                const long long row = static_cast<long long>(base) + static_cast<long long>(k) * step;
                mlq[q] = in ? __ldg(reinterpret_cast<const float2*>(rec_ml + row * ml_stride))
                            : make_float2(-INFINITY, 0.f);
                proj::RecRow<R>::load(rec_o + row * o_stride, lane, dc, in, v[q]);
            }
            float mq[kGemvRec];
            float mnew = mrun;
#pragma unroll
            for (int q = 0; q < kGemvRec; ++q) {   // an empty part (l = 0) contributes nothing
                mq[q] = mlq[q].y > 0.f ? mlq[q].x * mscale : -INFINITY;
                mnew = fmaxf(mnew, mq[q]);
            }
            if (mnew == -INFINITY) continue;
            const float sc = exp2f(mrun - mnew);
            lrun *= sc;
#pragma unroll
            for (int u4 = 0; u4 < 4; ++u4) {
                acc[u4].x *= sc; acc[u4].y *= sc; acc[u4].z *= sc; acc[u4].w *= sc;
            }
#pragma unroll
            for (int q = 0; q < kGemvRec; ++q) {
                float wq = exp2f(mq[q] - mnew);
                lrun = fmaf(wq, mlq[q].y, lrun);
                if (proj::RecRow<R>::kNormalised) wq *= mlq[q].y;   // an fp16 record holds o / l: weigh it by its row sum
#pragma unroll
                for (int u4 = 0; u4 < 4; ++u4) {
                    acc[u4].x = fmaf(wq, v[q][u4].x, acc[u4].x);
                    acc[u4].y = fmaf(wq, v[q][u4].y, acc[u4].y);
                    acc[u4].z = fmaf(wq, v[q][u4].z, acc[u4].z);
                    acc[u4].w = fmaf(wq, v[q][u4].w, acc[u4].w);
                }
            }
            mrun = mnew;
        }
        if (lane == 0) wml[warp] = make_float2(mrun, lrun);
#pragma unroll
        for (int u4 = 0; u4 < 4; ++u4) {
            const int c = proj::RecRow<R>::col(lane, u4);
            if (c < dc) *reinterpret_cast<float4*>(red + warp * dc + c) = acc[u4];
        }
    }
    return status0;
}

// Step 3 of the GEMV projection, shared by the projection kernels: thread (q, j) (4 quarters x dv
// rows, 512 threads) dots W_UV row j (128-byte-swizzled boxes in shared memory) with quarter q of
// every token's merged latent row olat[t], into qsum[q][t][j]; the caller sums the quarters in order.
template <typename T>
__device__ __forceinline__ void gemv_w_uv(const unsigned char* wsm, const float* olat, float* qsum, int B, int dc,
                                          int dv, bool ok) {
    const int q = threadIdx.x / dv, j = threadIdx.x % dv;   // 4 quarters x 128 rows
    const int kq = dc / 4;                                   // elements per quarter, a multiple of 16
    float acc[kGemvMaxTok] = {0.f, 0.f, 0.f, 0.f};
    if (ok) {
        for (int c = 0; c < kq / 8; ++c) {
            const int k = q * kq + 8 * c;
            // 128-byte-swizzled box row: 16-byte chunk ((k % 64) / 8) ^ (j % 8)
            const uint4 wv = *reinterpret_cast<const uint4*>(wsm + (k >> 6) * (dv * 128) + j * 128 +
                                                             ((((k & 63) >> 3) ^ (j & 7)) << 4));
            using T2 = typename ElemTraits<T>::T2;
            const float2 w01 = ElemTraits<T>::to_f2(*reinterpret_cast<const T2*>(&wv.x));
            const float2 w23 = ElemTraits<T>::to_f2(*reinterpret_cast<const T2*>(&wv.y));
            const float2 w45 = ElemTraits<T>::to_f2(*reinterpret_cast<const T2*>(&wv.z));
            const float2 w67 = ElemTraits<T>::to_f2(*reinterpret_cast<const T2*>(&wv.w));
#pragma unroll
            for (int tt = 0; tt < kGemvMaxTok; ++tt) {
                if (tt < B) {
                    const float4 o0 = *reinterpret_cast<const float4*>(olat + tt * dc + k);
                    const float4 o1 = *reinterpret_cast<const float4*>(olat + tt * dc + k + 4);
                    float a = acc[tt];
                    a = fmaf(w01.x, o0.x, a); a = fmaf(w01.y, o0.y, a);
                    a = fmaf(w23.x, o0.z, a); a = fmaf(w23.y, o0.w, a);
                    a = fmaf(w45.x, o1.x, a); a = fmaf(w45.y, o1.y, a);
                    a = fmaf(w67.x, o1.z, a); a = fmaf(w67.y, o1.w, a);
                    acc[tt] = a;
                }
            }
        }
    }
#pragma unroll
    for (int tt = 0; tt < kGemvMaxTok; ++tt)
        if (tt < B) qsum[(q * kGemvMaxTok + tt) * dv + j] = acc[tt];
}

template <typename T, typename R>
__global__ void __launch_bounds__(32 * kGemvWarps, 1)
project_gemv_kernel(const __grid_constant__ CUtensorMap tmap_w, const DecodePlan P, const float* __restrict__ rec_ml,
                    const R* __restrict__ rec_o, float* __restrict__ out, int parts, int ml_stride, int o_stride,
                    const PeerRows rows, const int* parity_epoch, size_t parity_elems) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const int dc = P.dc, dv = P.dv, B = P.B;   // dv == 128, dc % 64 == 0, dc <= 512, B <= kGemvMaxTok
    const int nk = dc / 64;
    unsigned char* wsm = smem;                                                    // nk x (dv rows x 128 B)
    float* red = reinterpret_cast<float*>(smem + nk * dv * 128);                  // [warp][dc]
    float2* wml = reinterpret_cast<float2*>(red + kGemvWarps * dc);               // [warp]
    float* olat = reinterpret_cast<float*>(wml + kGemvWarps);                     // [token][dc]
    float* qsum = olat + kGemvMaxTok * dc;                                        // [quarter][token][dv]
    uint64_t* bar = reinterpret_cast<uint64_t*>(qsum + 4 * kGemvMaxTok * dv);
    const uint32_t w_full = smem_u32(bar);

    const int h = blockIdx.x;
    const int wpt = kGemvWarps / B;
    volatile int* err = P.status;

    if (threadIdx.x == 0) {
        mbar_init(w_full, 1);
        fence_mbar_init();
        tma_prefetch_desc(&tmap_w);
        mbar_arrive_expect_tx(w_full, static_cast<uint32_t>(nk * dv * 128));
        for (int j = 0; j < nk; ++j) tma_load_2d(smem_u32(wsm) + j * dv * 128, &tmap_w, w_full, 64 * j, h * dv);
    }
    if (parity_epoch) {   // gathered partial sets: the half of the receive area the last step filled
        pdl_wait();       // the wait kernel before this one sets the step counter
        const size_t off = static_cast<size_t>(*parity_epoch & 1) * parity_elems;
        rec_ml += off;
        rec_o += off;
    }
    // ---- 1. merge
    const int status0 = gemv_merge<R>(P, rec_ml, rec_o, parts, ml_stride, o_stride, h, red, wml);
    __syncthreads();
    // ---- 2. per token: the warps' partials at the common max, summed in warp order
    for (int i = threadIdx.x; i < B * dc; i += blockDim.x) {
        const int tt = i / dc, c = i % dc;
        float M = -INFINITY;
        for (int w = tt * wpt; w < (tt + 1) * wpt; ++w) M = fmaxf(M, wml[w].x);
        float L = 0.f, o = 0.f;
        if (M != -INFINITY) {
            for (int w = tt * wpt; w < (tt + 1) * wpt; ++w) {
                const float a = wml[w].x == -INFINITY ? 0.f : exp2f(wml[w].x - M);
                L = fmaf(a, wml[w].y, L);
                o = fmaf(a, red[w * dc + c], o);
            }
        }
        olat[tt * dc + c] = L > 0.f ? o / L : 0.f;
    }
    // W_UV[h] must have landed (thread 0 waits; the block-wide AND carries the result)
    bool ok = true;
    // (a wait that ends only on completion or its time limit: the load never depends on another kernel)
    if (threadIdx.x == 0) ok = mbar_wait_impl<false, false>(w_full, 0, err, gcode(kSiteProjA), kDefaultWaitNs);
    ok = __syncthreads_and(ok);
    const bool failed = (parts == 0 && status0 != kStatusOk) || !ok;
    // ---- 3. thread (q, j): W_UV row j . latent quarter q, for every token
    gemv_w_uv<T>(wsm, olat, qsum, B, dc, dv, ok);
    __syncthreads();
    for (int i = threadIdx.x; i < B * dv; i += blockDim.x) {
        const int tt = i / dv, j = i % dv;
        float y = __int_as_float(0x7fc00000);   // a failed decode or wait shows in the output
        if (!failed)
            y = ((qsum[(0 * kGemvMaxTok + tt) * dv + j] + qsum[(1 * kGemvMaxTok + tt) * dv + j]) +
                 qsum[(2 * kGemvMaxTok + tt) * dv + j]) + qsum[(3 * kGemvMaxTok + tt) * dv + j];
        if (rows.world == 0) {
            out[(static_cast<long long>(tt) * P.H + h) * dv + j] = y;
        } else {
            // every rank's copy of the row (over NVLink for the peers)
            for (int q = 0; q < rows.world; ++q)
                reinterpret_cast<float*>(static_cast<unsigned char*>(rows.dst[q]) + rows.offset + tt * rows.pitch)
                    [h * dv + j] = y;
        }
    }
    if (rows.world > 0) peer_block_done_all(rows.sig, rows.world, gridDim.x);
    // shared memory is not released under a TMA write: if the wait gave up, wait (bounded) again
    if (threadIdx.x == 0 && !ok) mbar_wait_impl<false, false>(w_full, 0, err, gcode(kSiteProjA), 100000000ull);
}

// Partial export by the GEMV merge (B <= kGemvMaxTok): block h merges the decode's records of
// head h for every token and writes [m (natural log), l, 0, 0, o] with o the latent sum at the
// merged max, unnormalised (PartOut gives the place); a failed decode writes NaN into m and l.
// With part.peer the rows go to their slice's receiver, which is signalled by the last of the
// slice's H / slices blocks; with part.gather every rank receives every row, in the half of its
// receive area that the step's flag value selects, and is signalled by the last block.
template <typename T>
__global__ void __launch_bounds__(32 * kGemvWarps, 1)
export_gemv_kernel(const DecodePlan P, const float* __restrict__ rec_ml, const T* __restrict__ rec_o,
                   const PartOut part, const PeerSig sig) {
    extern __shared__ __align__(16) unsigned char smem_e[];
    const int dc = P.dc, B = P.B;
    float* red = reinterpret_cast<float*>(smem_e);                      // [warp][dc]
    float2* wml = reinterpret_cast<float2*>(red + kGemvWarps * dc);     // [warp]
    const int h = blockIdx.x;
    const int wpt = kGemvWarps / B;
    const int status0 = gemv_merge<T>(P, rec_ml, rec_o, 0, 2, dc, h, red, wml);
    __syncthreads();
    const bool failed = status0 != kStatusOk;
    const size_t half = part.gather ? static_cast<size_t>((*sig.epoch + 1) & 1) * part.parity_bytes : 0;
    for (int i = threadIdx.x; i < B * (dc + 4); i += blockDim.x) {
        const int tt = i / (dc + 4), c = i % (dc + 4) - 4;
        float M = -INFINITY;
        for (int w = tt * wpt; w < (tt + 1) * wpt; ++w) M = fmaxf(M, wml[w].x);
        float L = 0.f, o = 0.f;
        if (M != -INFINITY) {
            for (int w = tt * wpt; w < (tt + 1) * wpt; ++w) {
                const float a = wml[w].x == -INFINITY ? 0.f : exp2f(wml[w].x - M);
                L = fmaf(a, wml[w].y, L);
                if (c >= 0) o = fmaf(a, red[w * dc + c], o);
            }
        }
        float v = 0.f;   // the value of column c + 4 of the packed row ([m, l, 0, 0, o])
        if (c >= 0) v = o;
        else if (c == -4) v = failed ? __int_as_float(0x7fc00000) : (L > 0.f ? M * kLn2 : -INFINITY);
        else if (c == -3) v = failed ? __int_as_float(0x7fc00000) : L;
        if (part.gather) {
            const long long r = (static_cast<long long>(tt) * P.H + h) * (dc + 4) + (c + 4);
            for (int q = 0; q < part.gather; ++q)
                reinterpret_cast<float*>(static_cast<unsigned char*>(part.peer[q]) + part.peer_offset + half)[r] = v;
        } else if (c >= 0) {
            part.o_at(tt, h, B, P.H, dc)[c] = v;
        } else if (c <= -3 || part.slices) {   // m, l, and the packed row's padding
            part.ml_at(tt, h, B, P.H, dc)[c + 4] = v;
        }
    }
    if (part.gather) {
        peer_block_done_all(sig, part.gather, gridDim.x);
    } else if (part.to_peers()) {
        const int hs = P.H / part.slices;
        peer_block_done(sig, h / hs, static_cast<unsigned int>(hs));
    }
}

// ------------------------------------------------------------------------------------------
// One-kernel KV-range exchange (gathered form, B <= kGemvMaxTok)
// ------------------------------------------------------------------------------------------
constexpr int kLLMaxWorld = 64;
constexpr unsigned long long kLLWaitNs = 2000000000ull;   // 2 s

__device__ __forceinline__ void st_ll(unsigned char* p, float v0, float v1, int flag) {
    asm volatile("st.volatile.global.v4.b32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(__float_as_uint(v0)), "r"(flag),
                 "r"(__float_as_uint(v1)), "r"(flag)
                 : "memory");
}
// Spins (bounded) until both flags of the 16-byte unit at p equal `flag`; false when it gives up.
__device__ __forceinline__ bool ld_ll(const unsigned char* p, int flag, float& v0, float& v1) {
    const unsigned long long t0 = globaltimer_ns();
    while (true) {
        uint32_t a, f0, b, f1;
        asm volatile("ld.volatile.global.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(a), "=r"(f0), "=r"(b), "=r"(f1)
                     : "l"(p) : "memory");
        if (static_cast<int>(f0) == flag && static_cast<int>(f1) == flag) {
            v0 = __uint_as_float(a);
            v1 = __uint_as_float(b);
            return true;
        }
        if (globaltimer_ns() - t0 > kLLWaitNs) return false;
    }
}

// Block h of every rank: (1) merges the rank's decode records of head h (gemv_merge) into the packed
// partial [m (natural log), l, 0, 0, o] of each token, (2) stores it into every other rank's ring
// (NVLink stores) and keeps its own values in registers, (3) reads every other rank's partial of
// head h from its own ring (a bounded spin per 16-byte unit on the step's flag value), (4) merges the
// world partials in rank order and (5) projects with W_UV[h] (resident in shared memory, loaded at the
// start) into out. The last block advances the step counter. One kernel replaces the partial export,
// the wait and the merge of the gathered exchange; no fence is needed, since every value travels with
// its step. Every rank merges in rank order with the same code, so all ranks' outputs are equal bit
// for bit; against the NCCL path (the projection kernel's merge of partial sets) they differ in the
// last bits, where that merge rounds the log2 conversion differently.
template <typename T>
__global__ void __launch_bounds__(32 * kGemvWarps, 1)
exchange_merge_kernel(const __grid_constant__ CUtensorMap tmap_w, const DecodePlan P, const float* __restrict__ rec_ml,
                      const T* __restrict__ rec_o, float* __restrict__ out, const LLRing ring) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const int dc = P.dc, dv = P.dv, B = P.B, H = P.H;   // dv == 128, dc % 64 == 0, dc <= 512, B <= kGemvMaxTok
    const int nk = dc / 64, units = (dc + 4) / 2;        // 16-byte units of a ring row
    unsigned char* wsm = smem;                                                    // nk x (dv rows x 128 B)
    float* red = reinterpret_cast<float*>(smem + nk * dv * 128);                  // [warp][dc]
    float2* wml = reinterpret_cast<float2*>(red + kGemvWarps * dc);               // [warp]
    float* olat = reinterpret_cast<float*>(wml + kGemvWarps);                     // [token][dc]
    float* qsum = olat + kGemvMaxTok * dc;                                        // [quarter][token][dv]
    float2* mlp = reinterpret_cast<float2*>(qsum + 4 * kGemvMaxTok * dv);         // [rank][token] (m, l)
    float* wts = reinterpret_cast<float*>(mlp + kLLMaxWorld * kGemvMaxTok);      // [rank][token] weights
    float* ltot = wts + kLLMaxWorld * kGemvMaxTok;                                // [token]
    int* okw = reinterpret_cast<int*>(ltot + kGemvMaxTok);
    uint64_t* bar = reinterpret_cast<uint64_t*>(okw + 4);
    const uint32_t w_full = smem_u32(bar);
    const int h = blockIdx.x;
    const int wpt = kGemvWarps / B;
    const int world = ring.world, rank = ring.rank;
    volatile int* err = P.status;

    if (threadIdx.x == 0) {
        mbar_init(w_full, 1);
        fence_mbar_init();
        tma_prefetch_desc(&tmap_w);
        mbar_arrive_expect_tx(w_full, static_cast<uint32_t>(nk * dv * 128));
        for (int j = 0; j < nk; ++j) tma_load_2d(smem_u32(wsm) + j * dv * 128, &tmap_w, w_full, 64 * j, h * dv);
        okw[0] = 1;
    }
    const int e = *ring.epoch;   // written last by the previous step's kernel, which has ended
    const int flag = e + 1;
    const size_t half = static_cast<size_t>(flag & 1) * ring.half_bytes;
    // ---- 1. merge of this rank's records
    const int status0 = gemv_merge<T>(P, rec_ml, rec_o, 0, 2, dc, h, red, wml);
    __syncthreads();
    const bool failed = status0 != kStatusOk;
    // ---- 2. packed partials, unit u = columns 2u, 2u + 1, to every other rank; own values kept
    constexpr int kOwn = (kGemvMaxTok * 258 + 32 * kGemvWarps - 1) / (32 * kGemvWarps);
    float own[kOwn][2];
    {
        int k = 0;
        for (int i = threadIdx.x; i < B * units; i += blockDim.x, ++k) {
            const int tt = i / units, u = i % units;
            float M = -INFINITY;
            for (int w = tt * wpt; w < (tt + 1) * wpt; ++w) M = fmaxf(M, wml[w].x);
            float L = 0.f, o0 = 0.f, o1 = 0.f;
            const int c = 2 * u - 4;   // latent columns c, c + 1 (u >= 2)
            if (M != -INFINITY) {
                for (int w = tt * wpt; w < (tt + 1) * wpt; ++w) {
                    const float a = wml[w].x == -INFINITY ? 0.f : exp2f(wml[w].x - M);
                    L = fmaf(a, wml[w].y, L);
                    if (c >= 0) {
                        o0 = fmaf(a, red[w * dc + c], o0);
                        o1 = fmaf(a, red[w * dc + c + 1], o1);
                    }
                }
            }
            float v0 = o0, v1 = o1;
            if (u == 0) {
                const float nan = __int_as_float(0x7fc00000);
                v0 = failed ? nan : (L > 0.f ? M * kLn2 : -INFINITY);
                v1 = failed ? nan : L;
                mlp[rank * kGemvMaxTok + tt] = make_float2(v0, v1);
            } else if (u == 1) {
                v0 = v1 = 0.f;
            }
            if (k < kOwn) {
                own[k][0] = v0;
                own[k][1] = v1;
            }
            const size_t off = half + ((static_cast<size_t>(rank) * B + tt) * H + h) * units * 16 + u * 16;
            for (int q = 0; q < world; ++q)
                if (q != rank) st_ll(static_cast<unsigned char*>(ring.recv[q]) + off, v0, v1, flag);
        }
    }
    // ---- 3. (m, l) of every other rank's partials: thread p B + t reads unit 0 of row (p, t)
    const unsigned char* mine = static_cast<const unsigned char*>(ring.recv[rank]) + half;
    bool ok = true;
    for (int i = threadIdx.x; i < world * B; i += blockDim.x) {
        const int p = i / B, tt = i % B;
        if (p == rank) continue;
        float m = 0.f, l = 0.f;
        // after one wait gave up, the thread waits no more (a lost peer costs one bound, not many)
        if (ok && !ld_ll(mine + ((static_cast<size_t>(p) * B + tt) * H + h) * units * 16, flag, m, l)) ok = false;
        mlp[p * kGemvMaxTok + tt] = make_float2(m, l);
    }
    if (!ok) okw[0] = 0;
    __syncthreads();
    ok = okw[0] != 0;
    // ---- 4. per token: weights of the world partials (rank order), then the merged latent columns
    if (static_cast<int>(threadIdx.x) < B) {
        const int tt = threadIdx.x;
        // m in log2 units, rounded before the subtraction (no contraction into an FMA), so that every
        // rank weighs the partials alike
        float Mx = -INFINITY;
        for (int p = 0; p < world; ++p) {
            const float2 v = mlp[p * kGemvMaxTok + tt];
            if (v.y > 0.f) Mx = fmaxf(Mx, __fmul_rn(v.x, 1.4426950408889634f));
        }
        float L = 0.f;
        for (int p = 0; p < world; ++p) {
            const float2 v = mlp[p * kGemvMaxTok + tt];
            const float a =
                (v.y > 0.f && Mx != -INFINITY) ? exp2f(__fmul_rn(v.x, 1.4426950408889634f) - Mx) : 0.f;
            wts[p * kGemvMaxTok + tt] = a;
            L = fmaf(a, v.y, L);
        }
        ltot[tt] = L;
    }
    __syncthreads();
    {
        int k = 0;
        for (int i = threadIdx.x; i < B * units; i += blockDim.x, ++k) {
            const int tt = i / units, u = i % units;
            if (u < 2) continue;
            float o0 = 0.f, o1 = 0.f;
            for (int p = 0; p < world; ++p) {
                float v0 = 0.f, v1 = 0.f;
                if (p == rank) {
                    if (k < kOwn) {
                        v0 = own[k][0];
                        v1 = own[k][1];
                    }
                } else if (ok && !ld_ll(mine + ((static_cast<size_t>(p) * B + tt) * H + h) * units * 16 + u * 16, flag,
                                        v0, v1)) {
                    ok = false;
                }
                const float a = wts[p * kGemvMaxTok + tt];
                o0 = fmaf(a, v0, o0);
                o1 = fmaf(a, v1, o1);
            }
            const float L = ltot[tt];
            olat[tt * dc + 2 * u - 4] = L > 0.f ? o0 / L : 0.f;
            olat[tt * dc + 2 * u - 3] = L > 0.f ? o1 / L : 0.f;
        }
    }
    if (!ok) okw[0] = 0;
    // W_UV[h] must have landed (thread 0 waits; the block-wide AND carries the result)
    bool wok = true;
    if (threadIdx.x == 0) wok = mbar_wait_impl<false, false>(w_full, 0, err, gcode(kSiteProjA), kDefaultWaitNs);
    wok = __syncthreads_and(wok);
    const bool ring_ok = okw[0] != 0;
    if (!ring_ok && threadIdx.x == 0) atomicExch(ring.status, 1);
    // ---- 5. W_UV projection
    gemv_w_uv<T>(wsm, olat, qsum, B, dc, dv, wok);
    __syncthreads();
    for (int i = threadIdx.x; i < B * dv; i += blockDim.x) {
        const int tt = i / dv, j = i % dv;
        float y = __int_as_float(0x7fc00000);   // a failed decode, exchange or wait shows in the output
        if (wok && ring_ok)
            y = ((qsum[(0 * kGemvMaxTok + tt) * dv + j] + qsum[(1 * kGemvMaxTok + tt) * dv + j]) +
                 qsum[(2 * kGemvMaxTok + tt) * dv + j]) + qsum[(3 * kGemvMaxTok + tt) * dv + j];
        out[(static_cast<long long>(tt) * H + h) * dv + j] = y;
    }
    // the step counter moves once every block has read it
    if (threadIdx.x == 0) {
        const unsigned int prev = atomicAdd(ring.done, 1u);
        if (prev + 1u == gridDim.x) {
            *ring.done = 0u;
            *ring.epoch = flag;
        }
    }
    // shared memory is not released under a TMA write: if the wait gave up, wait (bounded) again
    if (threadIdx.x == 0 && !wok) mbar_wait_impl<false, false>(w_full, 0, err, gcode(kSiteProjA), 100000000ull);
}

bool absorb_sm100_supported(const DecodePlan& P) {
    return P.dn == 128 && P.dc % 256 == 0 && P.dc <= 512 && P.dR % 16 == 0 && P.dR <= 64;
}

bool project_sm100_supported(const DecodePlan& P) {
    return P.dv == 128 && P.dc % 64 == 0 && P.dc <= 512 && P.W <= 128;
}

// Largest batch absorbed, merged and projected by the fp32 GEMV kernels (LATENT_ATTN_B200_GEMV_TOKENS =
// 0 .. 4 overrides; 0 sends every batch to the tensor-core kernels).
int gemv_max_tokens() {
    static int v = [] {
        const char* s = std::getenv("LATENT_ATTN_B200_GEMV_TOKENS");
        if (!s) return kGemvMaxTok;
        const int n = std::atoi(s);
        return n < 0 ? 0 : (n > kGemvMaxTok ? kGemvMaxTok : n);
    }();
    return v;
}

// SM count of the current device (cached per device).
int sm_count() {
    static std::mutex mu;
    static std::vector<int> cache;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    std::lock_guard<std::mutex> lk(mu);
    if (static_cast<int>(cache.size()) <= dev) cache.resize(dev + 1, 0);
    if (cache[dev] == 0 && cudaDeviceGetAttribute(&cache[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        cache[dev] = 0;
    return cache[dev];
}

template <typename T>
cudaError_t launch_absorb_sm100(const DecodePlan& P, const float* q_nope, const T* W_UK, const float* q_rope,
                                float q_scale, T* qpack, int* tile_prefix_out, cudaStream_t s) {
    if (!absorb_sm100_supported(P)) return cudaErrorInvalidValue;
    if (P.B <= gemv_max_tokens()) {
        const cudaError_t e = launch_ex(absorb_gemv_kernel<T>, dim3(P.dc / kAbsorbGemvCols, P.H), dim3(256), 0, s, false,
                                        P, q_nope, W_UK, q_rope, q_scale, qpack, tile_prefix_out);
        count_launches(1);
        return e != cudaSuccess ? e : cudaGetLastError();
    }
    CUtensorMap tmap;
    if (!make_tmap_2d_16b(&tmap, W_UK, static_cast<uint64_t>(P.H) * P.dn, static_cast<uint64_t>(P.dc),
                          static_cast<uint64_t>(P.dc), static_cast<uint32_t>(P.dn), 64))
        return cudaErrorInvalidValue;
    const size_t smem = 1024 + absorb_smem_bytes(P.dn, P.dc);
    cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(absorb_sm100_kernel<T>), static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    dim3 grid(ceil_div(P.B, kAbsorbTok), P.H);
    e = launch_ex(absorb_sm100_kernel<T>, grid, dim3(kAbsorbThreads), smem, s, false, tmap, P, q_nope, q_rope, q_scale,
                  qpack, tile_prefix_out);
    count_launches(1);
    return e != cudaSuccess ? e : cudaGetLastError();
}

template <typename T, typename R>
cudaError_t launch_project_impl(const DecodePlan& P, const float* rec_ml, const R* rec_o, const T* W_UV,
                                float* out, bool pdl, int parts, int ml_stride, int o_stride, const PeerRows& rows,
                                cudaStream_t s, const int* parity_epoch = nullptr, size_t parity_elems = 0) {
    CUtensorMap tmap;
    if (!make_tmap_2d_16b(&tmap, W_UV, static_cast<uint64_t>(P.H) * P.dv, static_cast<uint64_t>(P.dc),
                          static_cast<uint64_t>(P.dc), static_cast<uint32_t>(P.dv), 64))
        return cudaErrorInvalidValue;
    if (P.B <= gemv_max_tokens() || (parity_epoch && P.B <= kGemvMaxTok)) {
        const size_t smem = 1024 + gemv_smem_bytes(P.dc, P.dv);
        cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(project_gemv_kernel<T, R>), static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        e = launch_ex(project_gemv_kernel<T, R>, dim3(P.H), dim3(32 * kGemvWarps), smem, s, pdl, tmap, P, rec_ml, rec_o,
                      out, parts, ml_stride, o_stride, rows, parity_epoch, parity_elems);
        count_launches(1);
        return e != cudaSuccess ? e : cudaGetLastError();
    }
    if (parity_epoch) return cudaErrorInvalidValue;   // gathered sets: B <= kGemvMaxTok only
    const int ntp = pad16(P.B < kProjTok ? P.B : kProjTok);
    const size_t smem = 1024 + proj::unit_smem_bytes(P.dc, P.dv, ntp) + 64;
    cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(project_sm100_kernel<T, R>), static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    dim3 grid(ceil_div(P.B, kProjTok), P.H);
    e = launch_ex(project_sm100_kernel<T, R>, grid, dim3(32 * kProjWarps), smem, s, pdl, tmap, P, rec_ml, rec_o, out, ntp,
                  tmem_cols_for(ntp), parts, ml_stride, o_stride, sm_count());
    count_launches(1);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess || rows.world == 0) return e;
    // the tensor-core kernel stages the rows in `out`; a put kernel sends them to every rank
    const size_t row_bytes = static_cast<size_t>(P.H) * P.dv * sizeof(float);
    const int blocks = static_cast<int>(std::min<size_t>(32, (static_cast<size_t>(P.B) * row_bytes + 16383) / 16384));
    return launch_peer_put(out, P.B, row_bytes, row_bytes, 0, rows.dst, rows.pitch, rows.offset, rows.world, blocks,
                           rows.sig, s);
}

template <typename T>
cudaError_t launch_project_sm100(const DecodePlan& P, const float* rec_ml, const T* rec_o, const T* W_UV,
                                 float* out, bool pdl, cudaStream_t s) {
    if (!project_sm100_supported(P)) return cudaErrorInvalidValue;
    return launch_project_impl<T, T>(P, rec_ml, rec_o, W_UV, out, pdl, 0, 2, P.dc, PeerRows{}, s);
}

// Status word of the partial-set merge: that path has no decode status to check, but the
// kernel's bounded waits need somewhere to record a timeout. Never read.
static __device__ int g_parts_status;

bool project_parts_sm100_supported(int H, int dc, int dv, int parts) {
    return dv == 128 && dc % 64 == 0 && dc <= 512 && parts >= 1 && parts <= 128 && H >= 1;
}

template <typename T>
cudaError_t launch_project_parts_sm100(int B, int H, int dc, int dv, int parts, const float* part_ml,
                                       const float* part_o, int ml_stride, int o_stride, const T* W_UV, float* out,
                                       const PeerRows& rows, cudaStream_t s, const int* parity_epoch,
                                       size_t parity_elems) {
    if (!project_parts_sm100_supported(H, dc, dv, parts)) return cudaErrorInvalidValue;
    static std::mutex mu;
    static std::vector<int*> status_addr;  // per device
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    int* status = nullptr;
    {
        std::lock_guard<std::mutex> lk(mu);
        if (static_cast<int>(status_addr.size()) <= dev) status_addr.resize(dev + 1, nullptr);
        if (!status_addr[dev]) {
            void* a = nullptr;
            e = cudaGetSymbolAddress(&a, g_parts_status);
            if (e != cudaSuccess) return e;
            status_addr[dev] = static_cast<int*>(a);
        }
        status = status_addr[dev];
    }
    DecodePlan P{};
    P.dc = dc;
    P.dv = dv;
    P.H = H;
    P.B = B;
    P.head_blocks = ceil_div(H, kGroupRows);
    P.status = status;
    // gathered sets follow the exchange's wait kernel, which lets this kernel start (and stream its
    // W_UV rows) while it waits
    return launch_project_impl<T, float>(P, part_ml, part_o, W_UV, out, parity_epoch != nullptr, parts, ml_stride,
                                         o_stride, rows, s, parity_epoch, parity_elems);
}

bool export_gemv_supported(const DecodePlan& P, bool gather) {
    return P.B >= 1 && P.B <= (gather ? kGemvMaxTok : gemv_max_tokens()) && P.dc % 64 == 0 && P.dc <= 512;
}

template <typename T>
cudaError_t launch_export_gemv(const DecodePlan& P, const float* rec_ml, const T* rec_o, const PartOut& part,
                               const PeerSig& sig, bool pdl, cudaStream_t s) {
    if (!export_gemv_supported(P, part.gather > 0)) return cudaErrorInvalidValue;
    const size_t smem = static_cast<size_t>(kGemvWarps) * P.dc * sizeof(float) + kGemvWarps * sizeof(float2);
    cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(export_gemv_kernel<T>), static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    e = launch_ex(export_gemv_kernel<T>, dim3(P.H), dim3(32 * kGemvWarps), smem, s, pdl, P, rec_ml, rec_o, part, sig);
    count_launches(1);
    return e != cudaSuccess ? e : cudaGetLastError();
}

size_t exchange_merge_smem_bytes(int dc, int dv) {
    return 1024 + gemv_smem_bytes(dc, dv) + static_cast<size_t>(kLLMaxWorld) * kGemvMaxTok * (sizeof(float2) + 4) +
           kGemvMaxTok * 4 + 16 + 16;
}

template <typename T>
cudaError_t launch_exchange_merge(const DecodePlan& P, const float* rec_ml, const T* rec_o, const T* W_UV,
                                  float* out, const LLRing& ring, cudaStream_t s) {
    if (P.B < 1 || P.B > kGemvMaxTok || P.dv != 128 || P.dc % 64 != 0 || P.dc > 512 || ring.world < 1 ||
        ring.world > kLLMaxWorld || ring.rank < 0 || ring.rank >= ring.world)
        return cudaErrorInvalidValue;
    CUtensorMap tmap;
    if (!make_tmap_2d_16b(&tmap, W_UV, static_cast<uint64_t>(P.H) * P.dv, static_cast<uint64_t>(P.dc),
                          static_cast<uint64_t>(P.dc), static_cast<uint32_t>(P.dv), 64))
        return cudaErrorInvalidValue;
    const size_t smem = exchange_merge_smem_bytes(P.dc, P.dv);
    cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(exchange_merge_kernel<T>), static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    e = launch_ex(exchange_merge_kernel<T>, dim3(P.H), dim3(32 * kGemvWarps), smem, s, true, tmap, P, rec_ml, rec_o,
                  out, ring);
    count_launches(1);
    return e != cudaSuccess ? e : cudaGetLastError();
}

#define MLA_INST(T)                                                                                              \
    template cudaError_t launch_absorb_sm100<T>(const DecodePlan&, const float*, const T*, const float*, float, T*, \
                                                int*, cudaStream_t);                                             \
    template cudaError_t launch_project_sm100<T>(const DecodePlan&, const float*, const T*, const T*, float*,       \
                                                 bool, cudaStream_t);                                             \
    template cudaError_t launch_project_parts_sm100<T>(int, int, int, int, int, const float*, const float*, int, int, \
                                                       const T*, float*, const PeerRows&, cudaStream_t,           \
                                                       const int*, size_t);                                         \
    template cudaError_t launch_export_gemv<T>(const DecodePlan&, const float*, const T*, const PartOut&,         \
                                               const PeerSig&, bool, cudaStream_t);                           \
    template cudaError_t launch_exchange_merge<T>(const DecodePlan&, const float*, const T*, const T*, float*,    \
                                                  const LLRing&, cudaStream_t);
MLA_INST(__half)
MLA_INST(__nv_bfloat16)
#undef MLA_INST

}  // namespace mla
