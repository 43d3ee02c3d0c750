// Building blocks of the split-KV merge + W_UV projection of one unit (up to kProjTok tokens of
// one head h), used by the projection kernel (gemm_sm100.cu):
//   out[b, h, :] = merge_k(records of (b, h)) . W_UV[h]^T        (src/fused_mla.cu:258-267)
// computed transposed, D^T[dv x tokens] = W_UV_h . o_lat^T with M = dv = 128 in TMEM:
//   A = W_UV_h, K-major, the d_c / 64 TMA boxes (64 columns x dv rows, 128-byte swizzle)
//   B = o_lat^T, K-major, 128-byte swizzle, written by the merge (rounded once to T)
// Records: see mla_internal.cuh (16-bit rows of the decode kernel) and RecRow<float> (the fp32
// partial sets of mla_decode_partial).
#pragma once
#include "mla_internal.cuh"
#include "sm100_ptx.cuh"

namespace mla {
namespace proj {
using namespace sm100;

constexpr int kProjTok = 64;       // tokens per unit (MMA N)
constexpr int kProjRedMax = 32;    // the largest red_rows
// rows of split partial sums of the merge (S * ntok <= rows): 32 when the token operand is at most
// 16 rows (32 merge jobs), else 8, which keeps the largest configuration inside the shared-memory limit
__host__ __device__ constexpr int red_rows(int ntp) { return ntp <= 16 ? 32 : 8; }

template <typename T> struct Fmt;
template <> struct Fmt<__half> { static constexpr uint32_t v = 0; };
template <> struct Fmt<__nv_bfloat16> { static constexpr uint32_t v = 1; };

template <typename T>
__device__ __forceinline__ uint32_t pack(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack<__half>(float a, float b) {
    __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
}
template <>
__device__ __forceinline__ uint32_t pack<__nv_bfloat16>(float a, float b) {
    __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ void sts_v2(uint32_t addr, uint32_t a, uint32_t b) {
    asm volatile("st.shared.v2.b32 [%0], {%1,%2};" ::"r"(addr), "r"(a), "r"(b) : "memory");
}
// AND of `pred` over the `nthreads` threads (whole warps) that reach named barrier `id`.
__device__ __forceinline__ bool bar_and(int id, int nthreads, bool pred) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "barrier.red.and.pred q, %2, %3, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"(static_cast<uint32_t>(pred)), "r"(id), "r"(nthreads)
        : "memory");
    return r != 0;
}
// Loads of records (written by an earlier kernel): the non-coherent path.
template <typename V>
__device__ __forceinline__ V ld_rec(const V* p) {
    return __ldg(p);
}

// Per-token record lists (records are read straight from global memory / L2).
struct alignas(16) Lists {        // size a multiple of 16: the float4 scratch and mbarriers follow it
    int cnt[kProjTok];            // records of token t
    int base[kProjTok];           // row of token t's first record; record k is at row base + k * step
    uint32_t valid[kProjTok][4];  // bit k: record k exists (a worker that owns no tile of the group wrote none)
    float2 split_ml[kProjRedMax]; // per (split, token) job: running max (log2 units) and row sum
    float split_w[kProjRedMax];   // per (split, token): weight of the split's sum in the token's row
};

// Shared memory of a unit, from a 1024-byte aligned base: W_UV_h, the B operand, the lists, the
// split partial sums, two mbarriers.
__host__ __device__ inline size_t unit_smem_bytes(int dc, int dv, int ntp) {
    return static_cast<size_t>(dc / 64) * dv * 128 + static_cast<size_t>(dc / 64) * ntp * 128 + sizeof(Lists) +
           static_cast<size_t>(red_rows(ntp)) * dc * sizeof(float) + 16;
}

// Records of (token b, head h): n rows starting at `base`, `step` rows apart (decode records: the
// workers w0 .. w0 + n - 1 that own tiles of the token's group; partial sets: all `parts` of them).
__device__ __forceinline__ void record_list(const DecodePlan& P, int b, int h, int parts, int ntiles, int& n, int& w0,
                                            int& base) {
    n = parts;
    w0 = 0;
    base = b * P.H + h;
    if (parts) return;
    int g, r;
    if (P.shared) {
        const int f = b * P.H + h;
        g = f / kGroupRows;
        r = f % kGroupRows;
    } else {
        g = b * P.head_blocks + h / kGroupRows;
        r = h % kGroupRows;
    }
    const int gt0 = tile_prefix(P, g), gt1 = tile_prefix(P, g + 1);
    n = 0;
    if (gt1 > gt0 && ntiles > 0) {
        w0 = worker_of_tile(ntiles, P.W, gt0);
        n = worker_of_tile(ntiles, P.W, gt1 - 1) - w0 + 1;
    }
    base = (g + w0) * kGroupRows + r;
}

// A lane's 16 elements of a partial row, as four float4 groups at columns col(lane, g):
//   fp32 rows (the caller's partial sets, unnormalised): float4 unit lane + 32 g, i.e. columns 4 (lane + 32 g) ..;
//   16-bit rows (the decode kernel's records, o or o / l by RecNorm): 16-byte unit lane + 32 (g / 2), i.e. columns
//   8 (lane + 32 (g / 2)) + 4 (g % 2) ...
// Rows hold d_c <= 512 elements; groups past d_c read as zeros.
template <typename R> struct RecRow {
    static constexpr bool kNormalised = RecNorm<R>::value;   // o / l (fp16 records of the decode kernel)
    __device__ static int col(int lane, int g) { return 8 * (lane + 32 * (g >> 1)) + 4 * (g & 1); }
    __device__ static void load(const R* row, int lane, int dc, bool in, float4 (&v)[4]) {
        using T2 = typename ElemTraits<R>::T2;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            const int c = 8 * (lane + 32 * hh);
            uint4 x = make_uint4(0u, 0u, 0u, 0u);
            if (in && c < dc) x = ld_rec(reinterpret_cast<const uint4*>(row + c));
            const float2 a = ElemTraits<R>::to_f2(*reinterpret_cast<const T2*>(&x.x));
            const float2 b = ElemTraits<R>::to_f2(*reinterpret_cast<const T2*>(&x.y));
            const float2 cc = ElemTraits<R>::to_f2(*reinterpret_cast<const T2*>(&x.z));
            const float2 d = ElemTraits<R>::to_f2(*reinterpret_cast<const T2*>(&x.w));
            v[2 * hh] = make_float4(a.x, a.y, b.x, b.y);
            v[2 * hh + 1] = make_float4(cc.x, cc.y, d.x, d.y);
        }
    }
};
template <> struct RecRow<float> {
    static constexpr bool kNormalised = false;  // unnormalised o (partial sets of mla_decode_partial)
    __device__ static int col(int lane, int g) { return 4 * (lane + 32 * g); }
    __device__ static void load(const float* row, int lane, int dc, bool in, float4 (&v)[4]) {
#pragma unroll
        for (int g = 0; g < 4; ++g) {
            const int c = 4 * (lane + 32 * g);
            v[g] = (in && c < dc) ? ld_rec(reinterpret_cast<const float4*>(row + c))
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
};

// Record lists of tokens b0 .. b0 + ntok - 1 of head h (thread t builds token t's list: the record
// count and first row are a few integer divisions; with every worker busy, or for partial sets,
// record k exists for every k < n). The caller synchronises the block afterwards.
__device__ __forceinline__ void build_lists(const DecodePlan& P, Lists* L, int b0, int ntok, int h, int parts,
                                            int ntiles) {
    const bool all_workers_busy = ntiles >= P.W;
    for (int t = threadIdx.x; t < ntok; t += blockDim.x) {
        int n, w0, base;
        record_list(P, b0 + t, h, parts, ntiles, n, w0, base);
        for (int c = 0; c < 4; ++c) {  // bit k % 32 of word k / 32: record k exists (n <= 128)
            uint32_t mask = 0u;
            const int k0 = 32 * c;
            if (parts || all_workers_busy) {
                const int m = n - k0;
                mask = m >= 32 ? 0xffffffffu : (m > 0 ? (1u << m) - 1u : 0u);
            } else {
                for (int k = k0; k < n && k < k0 + 32; ++k)
                    if (worker_begin(ntiles, P.W, w0 + k) != worker_begin(ntiles, P.W, w0 + k + 1))
                        mask |= 1u << (k - k0);
            }
            L->valid[t][c] = mask;
        }
        L->cnt[t] = n;
        L->base[t] = base;
    }
}

// Merge into the B operand (fp32 sums, rounded once to T) of ntp rows at b_u32; rows ntok .. ntp - 1
// are zero. Job p = (token p % ntok, record split p / ntok) takes the records s, s + S, ... of the
// token, lane l holding the four float4 groups RecRow<R>::col(l, 0..3) of the d_c row. A warp
// carries two jobs at once and loads the (m, l) pair and the o row of two records of each in one
// round trip, folding them into a running log-sum-exp (max, row sum, rescaled o sum). With few
// tokens the records of a token are split over S jobs (32 jobs in all), whose partial sums are
// rescaled to the common max and added through shared memory. Every thread of the block calls it.
template <typename T, typename R, int kWarps>
__device__ __forceinline__ void merge(const DecodePlan& P, Lists* L, float* red, uint32_t b_u32, int ntok, int ntp,
                                      int parts, int ml_stride, int o_stride, const float* __restrict__ rec_ml,
                                      const R* __restrict__ rec_o) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int dc = P.dc;
    const int step = parts ? P.B * P.H : kGroupRows;          // rows between a token's consecutive records
    const float mscale = parts ? 1.4426950408889634f : 1.f;   // m in log2 units
    const int U = dc / 4;                                      // float4 units per row, <= 128
    int S = red_rows(ntp) / ntok;
    S = S < 1 ? 1 : S;
    auto store_b = [&](int t, int c, float4 v) {   // columns c .. c + 3 of token t
        const uint32_t dst = b_u32 + (c >> 6) * (ntp * 128) + t * 128 + ((((c & 63) >> 3) ^ (t & 7)) << 4) +
                             ((c & 7) >> 2) * 8;
        sts_v2(dst, pack<T>(v.x, v.y), pack<T>(v.z, v.w));
    };
    const float4 zero4 = make_float4(0.f, 0.f, 0.f, 0.f);
    const int njobs = ntok * S;
    for (int p0 = warp; p0 < njobs; p0 += 2 * kWarps) {
        int tj[2], sj[2], nj[2], basej[2];
        const uint32_t* vmask[2];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int p = p0 + j * kWarps;
            const bool on = p < njobs;
            tj[j] = on ? p % ntok : 0;
            sj[j] = on ? p / ntok : 0;
            nj[j] = on ? L->cnt[tj[j]] : 0;
            basej[j] = L->base[tj[j]];
            vmask[j] = L->valid[tj[j]];
        }
        float mrun[2] = {-INFINITY, -INFINITY}, lrun[2] = {0.f, 0.f};
        float4 acc[2][4];
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
            for (int u = 0; u < 4; ++u) acc[j][u] = zero4;
        for (int i = 0;; i += 2) {
            bool more = false;
            long long rq[2][2];
            bool vq[2][2];
#pragma unroll
            for (int j = 0; j < 2; ++j)
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                    // record kk of the token: row base + kk * step; a missing record is never read
                    const int kk = sj[j] + (i + q) * S;
                    more |= kk < nj[j];
                    rq[j][q] = static_cast<long long>(basej[j]) + static_cast<long long>(kk) * step;
                    vq[j][q] = kk < nj[j] && ((vmask[j][kk >> 5] >> (kk & 31)) & 1u);
                }
            if (!more) break;
            float2 mlq[2][2];
            float4 v[2][2][4];
#pragma unroll
            for (int j = 0; j < 2; ++j)
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                    mlq[j][q] = vq[j][q] ? ld_rec(reinterpret_cast<const float2*>(rec_ml + rq[j][q] * ml_stride))
                                         : make_float2(-INFINITY, 0.f);
                    RecRow<R>::load(rec_o + rq[j][q] * o_stride, lane, dc, vq[j][q], v[j][q]);
                }
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                float mq[2];
#pragma unroll
                for (int q = 0; q < 2; ++q)   // an empty part (l = 0) contributes nothing
                    mq[q] = mlq[j][q].y > 0.f ? mlq[j][q].x * mscale : -INFINITY;
                const float mnew = fmaxf(mrun[j], fmaxf(mq[0], mq[1]));
                if (mnew == -INFINITY) continue;   // nothing in this job yet
                const float sc = exp2f(mrun[j] - mnew);
                float w0 = exp2f(mq[0] - mnew), w1 = exp2f(mq[1] - mnew);
                mrun[j] = mnew;
                lrun[j] = fmaf(lrun[j], sc, fmaf(w0, mlq[j][0].y, w1 * mlq[j][1].y));
                if (RecRow<R>::kNormalised) {   // an fp16 record holds o / l: weigh it by its row sum
                    w0 *= mlq[j][0].y;
                    w1 *= mlq[j][1].y;
                }
#pragma unroll
                for (int u4 = 0; u4 < 4; ++u4) {
                    acc[j][u4].x = fmaf(acc[j][u4].x, sc, fmaf(w0, v[j][0][u4].x, w1 * v[j][1][u4].x));
                    acc[j][u4].y = fmaf(acc[j][u4].y, sc, fmaf(w0, v[j][0][u4].y, w1 * v[j][1][u4].y));
                    acc[j][u4].z = fmaf(acc[j][u4].z, sc, fmaf(w0, v[j][0][u4].z, w1 * v[j][1][u4].z));
                    acc[j][u4].w = fmaf(acc[j][u4].w, sc, fmaf(w0, v[j][0][u4].w, w1 * v[j][1][u4].w));
                }
            }
        }
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            if (p0 + j * kWarps >= njobs) continue;
            if (S == 1) {
                const float inv = lrun[j] > 0.f ? 1.f / lrun[j] : 0.f;
#pragma unroll
                for (int u4 = 0; u4 < 4; ++u4) {
                    const int c = RecRow<R>::col(lane, u4);
                    if (c < dc)
                        store_b(tj[j], c, make_float4(acc[j][u4].x * inv, acc[j][u4].y * inv, acc[j][u4].z * inv,
                                                      acc[j][u4].w * inv));
                }
            } else {
                const int row = sj[j] * ntok + tj[j];
#pragma unroll
                for (int u4 = 0; u4 < 4; ++u4) {
                    const int c = RecRow<R>::col(lane, u4);
                    if (c < dc) reinterpret_cast<float4*>(red)[row * U + c / 4] = acc[j][u4];
                }
                if (lane == 0) L->split_ml[row] = make_float2(mrun[j], lrun[j]);
            }
        }
    }
    if (S > 1) {
        __syncthreads();
        // per token: the splits' common max and final weights 2^(m_s - M) / sum_s 2^(m_s - M) l_s
        // (lane s of a warp takes split s; S <= 32)
        for (int t = warp; t < ntok; t += kWarps) {
            const float2 ml = lane < S ? L->split_ml[lane * ntok + t] : make_float2(-INFINITY, 0.f);
            float M = ml.x;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
            const float w = ml.x == -INFINITY ? 0.f : exp2f(ml.x - M);   // an empty split weighs 0
            float l = w * ml.y;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
            if (lane < S) L->split_w[lane * ntok + t] = l > 0.f ? w / l : 0.f;
        }
        __syncthreads();
        // weighted sum over the splits: four lanes per (token, unit), each taking every fourth
        // split, then two shuffles (ntok * U * 4 is a multiple of 64: whole warps take part)
        for (int i = threadIdx.x; i < ntok * U * 4; i += blockDim.x) {
            const int q = i & 3, tu = i >> 2, u = tu % U, t = tu / U;
            float4 a = zero4;
            for (int sp = q; sp < S; sp += 4) {
                const float w = L->split_w[sp * ntok + t];
                const float4 v = reinterpret_cast<float4*>(red)[(sp * ntok + t) * U + u];
                a.x = fmaf(w, v.x, a.x); a.y = fmaf(w, v.y, a.y); a.z = fmaf(w, v.z, a.z); a.w = fmaf(w, v.w, a.w);
            }
#pragma unroll
            for (int o = 1; o < 4; o <<= 1) {
                a.x += __shfl_xor_sync(0xffffffffu, a.x, o);
                a.y += __shfl_xor_sync(0xffffffffu, a.y, o);
                a.z += __shfl_xor_sync(0xffffffffu, a.z, o);
                a.w += __shfl_xor_sync(0xffffffffu, a.w, o);
            }
            if (q == 0) store_b(t, 4 * u, a);
        }
    }
    // padding token rows are zero
    for (int i = threadIdx.x; i < (ntp - ntok) * U; i += blockDim.x)
        store_b(ntok + i / U, 4 * (i % U), make_float4(0.f, 0.f, 0.f, 0.f));
}

// One thread: the unit's MMAs, D[tmem] = W_UV_h (a_u32) . B^T (b_u32), K = d_c.
template <typename T>
__device__ __forceinline__ void issue_mma(uint32_t tmem, uint32_t a_u32, uint32_t b_u32, int dc, int dv, int ntp) {
    const uint32_t idesc = idesc_f16(dv, ntp, Fmt<T>::v, false, false);
    for (int k = 0; k < dc / 16; ++k) {
        const uint64_t ad = smem_desc_sw128(a_u32 + (k >> 2) * (dv * 128) + (k & 3) * 32, 16, 1024);
        const uint64_t bd = smem_desc_sw128(b_u32 + (k >> 2) * (ntp * 128) + (k & 3) * 32, 16, 1024);
        mma_ss(tmem, ad, bd, idesc, k > 0 ? 1u : 0u);
    }
}

// Warps 4-7 (warp w reads TMEM lanes 32 (w - 4) .. + 31, i.e. output columns j < dv = 128): the
// unit's outputs, or NaN when !ok (a wait gave up or the decode failed).
__device__ __forceinline__ void store_out(const DecodePlan& P, uint32_t tmem, float* __restrict__ out, int b0,
                                          int ntok, int h, bool ok) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int j = 32 * (warp - 4) + lane;
    if (ok) {
        tc_fence_after();
        const uint32_t trow = tmem + (static_cast<uint32_t>(32 * (warp - 4)) << 16);
        for (int c0 = 0; c0 < ntok; c0 += 16) {
            uint32_t r[16];
            tmem_ld16_sync(trow + c0, r);
#pragma unroll
            for (int q = 0; q < 16; ++q) {
                const int n = c0 + q;
                if (n < ntok) out[(static_cast<long long>(b0 + n) * P.H + h) * P.dv + j] = __uint_as_float(r[q]);
            }
        }
    } else {
        for (int n = 0; n < ntok; ++n) out[(static_cast<long long>(b0 + n) * P.H + h) * P.dv + j] = __int_as_float(0x7fc00000);
    }
}

}  // namespace proj
}  // namespace mla
