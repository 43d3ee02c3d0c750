// Tensor-core split-KV MLA decode for sm_100a on CTA pairs (tcgen05 cta_group::2 MMAs).
//
// One worker = a cluster of two CTAs (a "pair") that streams a contiguous range of
// 128-position tiles (the stream-K split of mla_internal.cuh). The pair's MMAs are issued by
// one thread of the leader CTA (rank 0) and run on both SMs: the 128 query rows (heads) of a
// group form the M = 128 tile, split 64 / 64, so CTA r owns heads [64 r, 64 r + 64) of the
// group -- their Q rows, their score rows, their softmax, their P rows and their output rows.
// The B operand (the cache) is split by N between the two CTAs' shared memory:
//   score  S[128 x 128] = Q[128 x 576] . KV[128 x 576]^T   N = positions: CTA r supplies
//          the full 576-wide rows of positions [64 r, 64 r + 64) of the tile
//   latent O[128 x 512] += P[128 x 128] . C[128 x 512]     two MMAs of N = 256 latent
//          columns; in MMA n CTA r supplies columns [256 n + 128 r, + 128) of all 128 positions
// Every SM does half of each product and each CTA's score tile holds complete scores for its
// 64 heads, so the softmax needs no data from the other CTA. The two operand layouts cut the
// tile differently (whole rows for the score, column slices for the latent product), so each
// CTA reads its column slices of the tile a second time (from L2: the other CTA has just read
// the rows from HBM); every cache byte crosses HBM once for all 128 heads.
//
// Tensor memory per CTA (512 columns): S buffers 0-63 and 64-127 (64 heads x 128 positions,
// lanes 0-63 positions 0-63 and lanes 64-127 positions 64-127), O 128-383 (per N = 256 MMA,
// lanes 0-63 latent [0, 128) and lanes 64-127 [128, 256) of that MMA's columns).
// Shared memory per CTA: Q (9 chunks of 64 rows x 64 elements, 128-byte swizzle), a ring of
// 8 KB stages, two P buffers (64 rows x 128 positions) and the softmax exchange slots.
//
// Per tile i the ring carries, in the order the MMAs consume them:
//   the rope chunk (this CTA's 64 positions x 64 k_rope elements; rotated in place by the
//   transform warps), 8 latent chunks (64 positions x 64 latent), then the 8 value chunks of
//   tile i - 1 (32 positions x 128 latent: value chunk (n, kb) holds positions [32 kb, + 32)
//   of the CTA's column slice of MMA n).
// The latent and value chunks are loaded with the pair form of TMA (completion counted on the
// leader's barrier); the rope chunk with the single-CTA form (its own barrier, which the
// transform warps wait on). In the last tile of a sequence, value chunks past the end are not
// loaded, and the one chunk per MMA that straddles the end is loaded single-CTA and its rows
// past the end are zeroed by the softmax warps before they release P (a zero weight times an
// uninitialised value could still be NaN).
//
// Warp roles (256 threads per CTA):
//   warp 0      TMA producer (one lane)
//   warp 1      tensor-memory allocation (both CTAs); MMA issue (one lane of the leader)
//   warps 2-3   transform: rotate the rope chunk's 64 positions (thread = position) with the
//               caller's cos/sin tables or cos/sin computed on the fly (src/fused_mla.cu:34-54)
//   warps 4-7   softmax: thread = TMEM lane L: head 64 r + (L % 64), positions [64 (L / 64), + 64)
//               of the tile; the two threads of a head exchange their half maxima through
//               shared memory. Online softmax in log2 units (Q is pre-scaled by
//               softmax_scale * log2 e) with a lazy reference: it only moves when a tile's max
//               exceeds it by more than 8, which bounds P by 2^8; only then is O rescaled.
//               At a group end the same warps write the partial record.
// Every wait is bounded (mbar_wait*); on timeout the kernel records kStatusTimeout in
// P.status, unwinds, and the merge kernel turns the outputs into NaN.
#include <cfloat>

#include "mla_internal.cuh"
#include "sm100_ptx.cuh"
#include "tma_host.cuh"

namespace mla {
using namespace sm100;

namespace {

constexpr int kTile = 128;                 // positions per tile
constexpr int kNS = 15;                    // ring stages
constexpr int kChunk = 8192;               // one stage: 64 rows x 128 bytes
constexpr int kQBytes = 9 * kChunk;        // Q: 8 latent chunks + the rope chunk
constexpr int kPBytes = 2 * kChunk;        // one P buffer: positions 0-63 | 64-127
constexpr int kChunksPerTile = 17;         // rope + 8 latent + 8 value chunks
constexpr int kThreads = 256;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0, kColO = 128;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

enum : int { kWaitProducer = 1, kWaitTransform = 2, kWaitMma = 3, kWaitSoftS = 7, kWaitSoftX = 8, kWaitSoftPV = 9,
             kWaitDrain = 11, kWaitBound = 12 };

struct __align__(8) Barriers {
    uint64_t full[kNS];        // leader: a pair-loaded chunk landed in both CTAs
    uint64_t empty[kNS];       // both: the MMAs reading the stage are done
    uint64_t rope_full[2];     // both: this CTA's rope chunk of tile i landed (slot i & 1)
    uint64_t rope_ready[2];    // leader: both CTAs' rope chunks of tile i are rotated
    uint64_t vbound[2];        // both: this CTA's straddling value chunk of MMA n landed
    uint64_t q_full;           // leader: both CTAs' Q of the group landed
    uint64_t q_empty;          // both: the group's last score MMA is done (Q may be reloaded)
    uint64_t s_full[2];        // both: score of tile i done (slot i & 1)
    uint64_t s_free[2];        // leader: both CTAs' softmax warps read S slot i & 1
    uint64_t p_full[2];        // leader: both CTAs' P of tile i written (slot i & 1)
    uint64_t pv_done[2];       // both: latent MMAs of tile i done (slot i & 1)
    uint64_t o_free;           // leader: both CTAs read O out for a record
    uint64_t drain;            // leader: every MMA done
    // the 4 softmax warps' hand-over of half-row maxima (slot i & 1) and of row sums at a group
    // end: bounded waits, so a warp that gives up never leaves the others blocked
    uint64_t xmax_full[2];
    uint64_t xsum_full;
    uint32_t tmem_base;
};

constexpr size_t kOffQ = 0;
constexpr size_t kOffRing = kOffQ + kQBytes;
constexpr size_t kOffP = kOffRing + static_cast<size_t>(kNS) * kChunk;
constexpr size_t kOffX = kOffP + 2 * kPBytes;                  // xmax[2 slots][2 halves][64] floats
constexpr size_t kOffL = kOffX + 2 * 2 * 64 * sizeof(float);   // xsum[2 halves][64] floats
constexpr size_t kOffBars = kOffL + 2 * 64 * sizeof(float);
constexpr size_t kSmemBytes = kOffBars + sizeof(Barriers) + 1024;   // + alignment slack
static_assert(kSmemBytes <= 232448, "shared memory budget");

struct Maps {
    CUtensorMap kv;   // cache rows: box 64 rows x 64 columns, 128-byte swizzle
    CUtensorMap v;    // cache rows: box 32 rows x 64 columns, 128-byte swizzle (value chunks)
    CUtensorMap q;    // packed queries (G * 128 rows x 576): box 64 x 64, 128-byte swizzle
};

__device__ __forceinline__ int code(int site) { return kStatusTimeout | (site << 8); }

static __device__ __noinline__ void note_fail(volatile int* err, int site, int tile) {
    int* e = const_cast<int*>(err);
    atomicAdd(e + 1, 1);
    atomicCAS(e + 2, 0, ((static_cast<int>(blockIdx.x) + 1) << 16) | (tile & 0xFFFF));
    atomicOr(e + 3, 1 << site);
}

__device__ __forceinline__ bool warp_ok(bool ok) { return __all_sync(0xffffffffu, ok); }

// Walks the worker's tiles; every role advances an identical copy.
struct TileIter {
    int t, t_begin, t_end;
    int g, gt0, gt1, len;
    long long row0;

    __device__ void load_group(const DecodePlan& P) {
        gt0 = tile_prefix(P, g);
        gt1 = tile_prefix(P, g + 1);
        len = group_len(P, g);
        row0 = group_kv_row0(P, g);
    }
    __device__ void init(const DecodePlan& P, int tb, int te) {
        t = t_begin = tb;
        t_end = te;
        g = group_of_tile(P, tb);
        load_group(P);
    }
    __device__ bool valid() const { return t < t_end; }
    __device__ int pos0() const { return (t - gt0) * kTile; }
    __device__ int np() const { int r = len - pos0(); return r < kTile ? r : kTile; }
    __device__ bool seg_first() const { return t == t_begin || t == gt0; }
    __device__ bool seg_last() const { return t + 1 == t_end || t + 1 == gt1; }
    __device__ void next(const DecodePlan& P) {
        ++t;
        if (t < t_end && t >= gt1) {
            ++g;
            while (g < P.G - 1 && tile_prefix(P, g + 1) <= t) ++g;  // skip empty groups
            load_group(P);
        }
    }
};

// Chunk sequence of a worker with n tiles: iteration i < n carries the rope chunk and the 8
// latent chunks of tile i, then (i >= 1) the 8 value chunks of tile i - 1; iteration n carries
// only the value chunks of tile n - 1.
__device__ __forceinline__ int chunks_before(int i) { return i == 0 ? 0 : kChunksPerTile * i - 8; }
__device__ __forceinline__ int value_chunk0(int j, int n) { return chunks_before(j + 1) + (j + 1 < n ? 9 : 0); }

// Value chunk (n, kb) of a tile with np valid positions: 0 = past the end (not loaded, no MMA),
// 1 = straddles the end (single-CTA load, tail rows zeroed), 2 = complete (pair load).
__device__ __forceinline__ int vchunk_kind(int np, int kb) {
    const int lo = 32 * kb;
    return lo >= np ? 0 : (lo + 32 > np ? 1 : 2);
}

template <typename T> struct MmaFmt2;
template <> struct MmaFmt2<__half> { static constexpr uint32_t v = 0; };
template <> struct MmaFmt2<__nv_bfloat16> { static constexpr uint32_t v = 1; };

__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}
template <typename T>
__device__ __forceinline__ float2 unpack2(uint32_t v) {
    return ElemTraits<T>::to_f2(*reinterpret_cast<const typename ElemTraits<T>::T2*>(&v));
}

__device__ __forceinline__ void st_row32(float* p, const uint32_t (&v)[32]) {
#pragma unroll
    for (int q = 0; q < 4; ++q)
        asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p + 8 * q), "r"(v[8 * q]),
                     "r"(v[8 * q + 1]), "r"(v[8 * q + 2]), "r"(v[8 * q + 3]), "r"(v[8 * q + 4]), "r"(v[8 * q + 5]),
                     "r"(v[8 * q + 6]), "r"(v[8 * q + 7])
                     : "memory");
}

// Arrive on a barrier of the leader CTA: a local arrive in the leader, a cluster-scope release
// arrive from the other CTA (its earlier shared-memory writes become visible first).
__device__ __forceinline__ void arrive_leader(uint32_t local_bar, uint32_t rank) {
    if (rank == 0) mbar_arrive(local_bar);
    else mbar_arrive_remote(mapa(local_bar, 0));
}

// Cache row of the 64-position half starting at position pos (a multiple of 64) of group g:
// contiguous row0 + pos, or through the page table; -1 for a page outside the cache.
__device__ __forceinline__ long long half_row(const DecodePlan& P, int g, long long row0, int pos, bool paged) {
    if (!paged) return row0 + pos;
    return tile_kv_row(P, g, row0, pos);
}

}  // namespace

template <typename T, bool kPaged>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
decode_2sm_kernel(const __grid_constant__ Maps maps, const DecodePlan P, const float* __restrict__ cos_tab,
                  const float* __restrict__ sin_tab, float* __restrict__ rec_ml, float* __restrict__ rec_o) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    Barriers* bars = reinterpret_cast<Barriers*>(smem + kOffBars);
    float* xmax = reinterpret_cast<float*>(smem + kOffX);
    float* xsum = reinterpret_cast<float*>(smem + kOffL);
    const uint32_t sbase = smem_u32(smem);
    const uint32_t q_u32 = sbase + kOffQ, ring_u32 = sbase + kOffRing, p_u32 = sbase + kOffP;

    const uint32_t rank = cluster_ctarank();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int w = blockIdx.x >> 1;
    volatile int* err = P.status;

    if (threadIdx.x == 0) {
        pdl_launch_dependents();
        tma_prefetch_desc(&maps.kv);
        tma_prefetch_desc(&maps.v);
        tma_prefetch_desc(&maps.q);
    }
    // with variable lengths the tile prefix comes from the previous kernel
    const bool uniform = P.uniform_len > 0;
    if (!uniform) pdl_wait();
    const int ntiles = total_tiles(P);
    if (ntiles <= 0 || w >= P.W) return;  // identical for both CTAs of the pair
    const int tb = worker_begin(ntiles, P.W, w), te = worker_begin(ntiles, P.W, w + 1);
    if (tb >= te) return;
    const int n = te - tb;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kNS; ++s) {
            mbar_init(smem_u32(&bars->full[s]), 1);
            mbar_init(smem_u32(&bars->empty[s]), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(smem_u32(&bars->rope_full[b]), 1);
            mbar_init(smem_u32(&bars->rope_ready[b]), 4);   // 2 transform warps x 2 CTAs
            mbar_init(smem_u32(&bars->vbound[b]), 1);
            mbar_init(smem_u32(&bars->s_full[b]), 1);
            mbar_init(smem_u32(&bars->s_free[b]), 8);       // 4 softmax warps x 2 CTAs
            mbar_init(smem_u32(&bars->p_full[b]), 8);
            mbar_init(smem_u32(&bars->pv_done[b]), 1);
        }
        mbar_init(smem_u32(&bars->q_full), 1);
        mbar_init(smem_u32(&bars->q_empty), 1);
        mbar_init(smem_u32(&bars->o_free), 8);
        mbar_init(smem_u32(&bars->drain), 1);
        mbar_init(smem_u32(&bars->xmax_full[0]), 4);
        mbar_init(smem_u32(&bars->xmax_full[1]), 4);
        mbar_init(smem_u32(&bars->xsum_full), 4);
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc_pair(smem_u32(&bars->tmem_base), kTmemCols);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync();  // both CTAs: barriers initialised, tensor memory allocated
    tc_fence_after();
    const uint32_t tbase = bars->tmem_base;

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            const bool leader = rank == 0;
            TileIter it, iv;
            it.init(P, tb, te);
            iv = it;
            int c = 0, qgroups = 0;
            bool pdl_done = !uniform, bad_page = false, ok = true;
            auto acquire = [&](int cc) -> int {
                const int s = cc % kNS;
                if (cc >= kNS && !mbar_wait_cluster(smem_u32(&bars->empty[s]), ((cc / kNS) - 1) & 1, err,
                                                    code(kWaitProducer))) {
                    note_fail(err, kWaitProducer, cc);
                    ok = false;
                }
                return s;
            };
            for (int i = 0; ok && i <= n; ++i) {
                if (i < n) {
                    // this CTA's 64 positions of tile i
                    long long y = half_row(P, it.g, it.row0, it.pos0() + 64 * static_cast<int>(rank), kPaged);
                    if (y < 0) {
                        bad_page = true;
                        y = -2 * kTile;   // reads zeros
                    }
                    const int yi = static_cast<int>(y);
                    int s = acquire(c);
                    if (!ok) break;
                    const uint32_t rf = smem_u32(&bars->rope_full[i & 1]);
                    mbar_arrive_expect_tx(rf, kChunk);
                    tma_load_2d(ring_u32 + s * kChunk, &maps.kv, rf, P.dc, yi);
                    ++c;
                    for (int k = 0; k < 8; ++k) {
                        s = acquire(c);
                        if (!ok) break;
                        const uint32_t fb = smem_u32(&bars->full[s]);
                        if (leader) mbar_arrive_expect_tx(fb, 2 * kChunk);
                        tma_load_2d_pair(ring_u32 + s * kChunk, &maps.kv, mapa(fb, 0), 64 * k, yi);
                        ++c;
                    }
                    if (!ok) break;
                    if (it.seg_first()) {
                        // the group's Q, once the previous group's last score MMA has read the old one
                        if (qgroups > 0 &&
                            !mbar_wait_cluster(smem_u32(&bars->q_empty), (qgroups - 1) & 1, err, code(kWaitProducer))) {
                            note_fail(err, kWaitProducer, -1);
                            break;
                        }
                        if (!pdl_done) {
                            pdl_wait();  // the packed queries come from the previous kernel
                            pdl_done = true;
                        }
                        const uint32_t qb = smem_u32(&bars->q_full);
                        if (leader) mbar_arrive_expect_tx(qb, 2 * kQBytes);
                        const int qrow = it.g * kGroupRows + 64 * static_cast<int>(rank);
                        for (int k = 0; k < 9; ++k) tma_load_2d_pair(q_u32 + k * kChunk, &maps.q, mapa(qb, 0), 64 * k, qrow);
                        ++qgroups;
                    }
                    it.next(P);
                }
                if (i >= 1) {
                    // value chunks of tile i - 1: columns [256 n + 128 r, + 128), positions [32 kb, + 32)
                    const int np = iv.np();
                    long long yh[2];
                    for (int hh = 0; hh < 2; ++hh) {
                        yh[hh] = half_row(P, iv.g, iv.row0, iv.pos0() + 64 * hh, kPaged);
                        if (yh[hh] < 0) {
                            bad_page = true;
                            yh[hh] = -2 * kTile;
                        }
                    }
                    for (int nn = 0; nn < 2 && ok; ++nn) {
                        for (int kb = 0; kb < 4; ++kb) {
                            const int s = acquire(c);
                            if (!ok) break;
                            const int kind = vchunk_kind(np, kb);
                            const int x0 = 256 * nn + 128 * static_cast<int>(rank);
                            const int yv = static_cast<int>(yh[kb >> 1] + 32 * (kb & 1));
                            const uint32_t dst = ring_u32 + s * kChunk;
                            if (kind == 2) {
                                const uint32_t fb = smem_u32(&bars->full[s]);
                                if (leader) mbar_arrive_expect_tx(fb, 2 * kChunk);
                                tma_load_2d_pair(dst, &maps.v, mapa(fb, 0), x0, yv);
                                tma_load_2d_pair(dst + 4096, &maps.v, mapa(fb, 0), x0 + 64, yv);
                            } else if (kind == 1) {
                                const uint32_t vb = smem_u32(&bars->vbound[nn]);
                                mbar_arrive_expect_tx(vb, kChunk);
                                tma_load_2d(dst, &maps.v, vb, x0, yv);
                                tma_load_2d(dst + 4096, &maps.v, vb, x0 + 64, yv);
                            }
                            ++c;
                        }
                    }
                    iv.next(P);
                }
            }
            if (!pdl_done) pdl_wait();  // the status words may only be written after the previous kernel
            if (bad_page) atomicCAS(const_cast<int*>(err), 0, kStatusBadPage);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer (leader)
        if (rank == 0 && lane == 0) {
            constexpr uint32_t fmt = MmaFmt2<T>::v;
            constexpr uint32_t idesc_qk = idesc_f16(128, kTile, fmt, false, false);
            constexpr uint32_t idesc_pv = idesc_f16(128, 256, fmt, false, true);
            TileIter it, iv;
            it.init(P, tb, te);
            iv = it;
            int c = 0, qg = 0, vg = 0;
            uint32_t fbits = 0;
            bool ok = true;
            auto wait_full = [&](int s) -> bool {
                const bool got = mbar_wait_cluster(smem_u32(&bars->full[s]), (fbits >> s) & 1u, err, code(kWaitMma));
                fbits ^= 1u << s;
                if (!got) note_fail(err, kWaitMma, c);
                return got;
            };
            for (int i = 0; ok && i <= n; ++i) {
                if (i < n) {
                    // ---- score of tile i into S slot i & 1
                    if (it.seg_first()) {
                        ok = mbar_wait_cluster(smem_u32(&bars->q_full), qg & 1, err, code(kWaitMma));
                        ++qg;
                        if (!ok) { note_fail(err, kWaitMma, -2); break; }
                    }
                    if (i >= 2 && !(ok = mbar_wait_cluster(smem_u32(&bars->s_free[i & 1]), ((i - 2) >> 1) & 1, err,
                                                          code(kWaitMma)))) {
                        note_fail(err, kWaitMma, -3);
                        break;
                    }
                    const uint32_t tS = tbase + kColS + 64u * (i & 1);
                    const int s_rope = c % kNS;
                    ++c;
                    for (int k = 0; k < 8; ++k) {
                        const int s = c % kNS;
                        if (!(ok = wait_full(s))) break;
                        tc_fence_after();
                        const uint64_t ad = smem_desc_sw128(q_u32 + k * kChunk, 16, 1024);
                        const uint64_t bd = smem_desc_sw128(ring_u32 + s * kChunk, 16, 1024);
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk)
                            mma_ss_pair(tS, ad + static_cast<uint64_t>(2 * kk), bd + static_cast<uint64_t>(2 * kk),
                                        idesc_qk, (k | kk) != 0 ? 1u : 0u);
                        mma_commit_pair_both(smem_u32(&bars->empty[s]));
                        ++c;
                    }
                    if (!ok) break;
                    if (!(ok = mbar_wait_cluster(smem_u32(&bars->rope_ready[i & 1]), (i >> 1) & 1, err, code(kWaitMma)))) {
                        note_fail(err, kWaitMma, -4);
                        break;
                    }
                    tc_fence_after();
                    {
                        const uint64_t ad = smem_desc_sw128(q_u32 + 8 * kChunk, 16, 1024);
                        const uint64_t bd = smem_desc_sw128(ring_u32 + s_rope * kChunk, 16, 1024);
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk)
                            mma_ss_pair(tS, ad + static_cast<uint64_t>(2 * kk), bd + static_cast<uint64_t>(2 * kk),
                                        idesc_qk, 1u);
                    }
                    mma_commit_pair_both(smem_u32(&bars->empty[s_rope]));
                    mma_commit_pair_both(smem_u32(&bars->s_full[i & 1]));
                    if (it.seg_last()) mma_commit_pair_both(smem_u32(&bars->q_empty));
                    it.next(P);
                }
                if (i >= 1) {
                    // ---- latent product of tile j = i - 1
                    const int j = i - 1;
                    if (!(ok = mbar_wait_cluster(smem_u32(&bars->p_full[j & 1]), (j >> 1) & 1, err, code(kWaitMma)))) {
                        note_fail(err, kWaitMma, -5);
                        break;
                    }
                    const bool first = iv.seg_first();
                    if (first && vg > 0 &&
                        !(ok = mbar_wait_cluster(smem_u32(&bars->o_free), (vg - 1) & 1, err, code(kWaitMma)))) {
                        note_fail(err, kWaitMma, -6);
                        break;
                    }
                    tc_fence_after();
                    const int np = iv.np();
                    const uint32_t pbuf = p_u32 + (j & 1) * kPBytes;
                    for (int nn = 0; nn < 2 && ok; ++nn) {
                        const uint32_t tO = tbase + kColO + 128u * nn;
                        for (int kb = 0; kb < 4; ++kb) {
                            const int s = c % kNS;
                            const int kind = vchunk_kind(np, kb);
                            if (kind == 2) {
                                if (!(ok = wait_full(s))) break;
                                tc_fence_after();
                            }
                            if (kind != 0) {
                                const uint64_t vd = smem_desc_sw128(ring_u32 + s * kChunk, 4096, 1024);
#pragma unroll
                                for (int kk = 0; kk < 2; ++kk) {
                                    const int kpos = 32 * kb + 16 * kk;
                                    if (kpos < np) {
                                        const uint64_t pd =
                                            smem_desc_sw128(pbuf + (kpos >> 6) * kChunk + (kpos & 63) * 2, 16, 1024);
                                        mma_ss_pair(tO, pd, vd + static_cast<uint64_t>((2048 * kk) >> 4), idesc_pv,
                                                    (first && kpos == 0) ? 0u : 1u);
                                    }
                                }
                            }
                            mma_commit_pair_both(smem_u32(&bars->empty[s]));
                            ++c;
                        }
                    }
                    if (!ok) break;
                    mma_commit_pair_both(smem_u32(&bars->pv_done[j & 1]));
                    if (iv.seg_last()) ++vg;
                    iv.next(P);
                }
            }
            if (!ok) atomicCAS(const_cast<int*>(err), 0, code(kWaitMma));
            // every MMA this thread issued has completed before teardown
            mma_commit_pair(smem_u32(&bars->drain));
            mbar_wait(smem_u32(&bars->drain), 0, err, code(kWaitDrain));
        }
    } else if (warp < 4) {
        // ------------------------------------------------------------ rope transform
        const int p = threadIdx.x - 64;   // position within this CTA's half of the tile
        TileIter it;
        it.init(P, tb, te);
        const int half = P.dR / 2;        // 32
        for (int i = 0; it.valid(); ++i, it.next(P)) {
            const int pos_t = it.pos0() + 64 * static_cast<int>(rank) + p;
            const bool valid = pos_t < it.len;
            const long long pos = static_cast<long long>(P.kv_pos_offset) + pos_t;
            // the caller's table rows are read before the wait, so their latency overlaps it
            float4 tc[8], ts[8];
            if (valid && !P.rope_otf) {
                const float4* c4 = reinterpret_cast<const float4*>(cos_tab + pos * half);
                const float4* s4 = reinterpret_cast<const float4*>(sin_tab + pos * half);
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    tc[q] = __ldg(c4 + q);
                    ts[q] = __ldg(s4 + q);
                }
            }
            const bool got = mbar_wait(smem_u32(&bars->rope_full[i & 1]), (i >> 1) & 1, err, code(kWaitTransform));
            if (!warp_ok(got)) {
                if (!got) note_fail(err, kWaitTransform, i);
                break;
            }
            const int s = chunks_before(i) % kNS;
            unsigned char* row = smem + kOffRing + s * kChunk + p * 128;
            if (valid) {
                // logical 16-byte unit u of the row sits at unit u ^ (p % 8); pair (e, e + 32)
                // is element e % 8 of units e / 8 and e / 8 + 4
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    uint4* pa = reinterpret_cast<uint4*>(row + ((u ^ (p & 7)) << 4));
                    uint4* pb = reinterpret_cast<uint4*>(row + (((u + 4) ^ (p & 7)) << 4));
                    const uint4 ka = *pa, kb = *pb;
                    const uint32_t xa[4] = {ka.x, ka.y, ka.z, ka.w}, xb[4] = {kb.x, kb.y, kb.z, kb.w};
                    float cs[8], sn[8];
                    if (P.rope_otf) {
#pragma unroll
                        for (int e = 0; e < 8; ++e)
                            rope_sincos_exact(pos, P.rope_freq[8 * u + e], &sn[e], &cs[e]);
                    } else {
                        const float4 c0 = tc[2 * u], c1 = tc[2 * u + 1], s0 = ts[2 * u], s1 = ts[2 * u + 1];
                        cs[0] = c0.x; cs[1] = c0.y; cs[2] = c0.z; cs[3] = c0.w;
                        cs[4] = c1.x; cs[5] = c1.y; cs[6] = c1.z; cs[7] = c1.w;
                        sn[0] = s0.x; sn[1] = s0.y; sn[2] = s0.z; sn[3] = s0.w;
                        sn[4] = s1.x; sn[5] = s1.y; sn[6] = s1.z; sn[7] = s1.w;
                    }
                    uint32_t ya[4], yb[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float2 x0 = unpack2<T>(xa[e]), x1 = unpack2<T>(xb[e]);
                        const float c_lo = cs[2 * e], c_hi = cs[2 * e + 1], s_lo = sn[2 * e], s_hi = sn[2 * e + 1];
                        ya[e] = pack2<T>(x0.x * c_lo - x1.x * s_lo, x0.y * c_hi - x1.y * s_hi);
                        yb[e] = pack2<T>(x0.x * s_lo + x1.x * c_lo, x0.y * s_hi + x1.y * c_hi);
                    }
                    *pa = make_uint4(ya[0], ya[1], ya[2], ya[3]);
                    *pb = make_uint4(yb[0], yb[1], yb[2], yb[3]);
                }
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) arrive_leader(smem_u32(&bars->rope_ready[i & 1]), rank);
        }
    } else {
        // ------------------------------------------------------------ softmax + records
        const int L = threadIdx.x - 128;             // TMEM lane
        const int r = L & 63, hf = L >> 6;            // head row within the CTA's 64, position half
        const uint32_t tlane = tbase + (static_cast<uint32_t>(32 * (warp & 3)) << 16);
        TileIter it;
        it.init(P, tb, te);
        float m = 0.f, lh = 0.f;   // row reference (log2 units) and this half's row sum
        int nbound = 0;            // straddling value chunks waited for so far (phase of vbound)
        int nsum = 0;              // row-sum hand-overs so far (phase of xsum_full)
        bool ok = true;
        for (int j = 0; ok && it.valid(); ++j, it.next(P)) {
            bool got = mbar_wait_cluster(smem_u32(&bars->s_full[j & 1]), (j >> 1) & 1, err, code(kWaitSoftS));
            if (!warp_ok(got)) {
                if (!got) note_fail(err, kWaitSoftS, j);
                ok = false;
                break;
            }
            tc_fence_after();
            float s[64];
            {
                uint32_t sr[64];
                tmem_ld64_sync(tlane + kColS + 64u * (j & 1), sr);
#pragma unroll
                for (int k = 0; k < 64; ++k) s[k] = __uint_as_float(sr[k]);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) arrive_leader(smem_u32(&bars->s_free[j & 1]), rank);
            const int np = it.np();
            const int nv = np - 64 * hf;  // valid positions of this half
            if (nv < 64) {
#pragma unroll
                for (int k = 0; k < 64; ++k)
                    if (k >= nv) s[k] = -INFINITY;
            }
            float mx[32];
#pragma unroll
            for (int k = 0; k < 32; ++k) mx[k] = fmaxf(s[k], s[k + 32]);
#pragma unroll
            for (int w2 = 16; w2 > 0; w2 >>= 1)
#pragma unroll
                for (int k = 0; k < w2; ++k) mx[k] = fmaxf(mx[k], mx[k + w2]);
            // the row's max over both halves (the other half is lane L ^ 64, in warp w ^ 2). A slot's
            // next phase needs every warp's arrival for tile j + 2, which each warp makes only after
            // its own wait for tile j + 1, so the slot cannot complete two phases ahead of a waiter.
            xmax[((j & 1) * 2 + hf) * 64 + r] = mx[0];
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&bars->xmax_full[j & 1]));
            got = mbar_wait(smem_u32(&bars->xmax_full[j & 1]), (j >> 1) & 1, err, code(kWaitSoftX));
            if (!warp_ok(got)) {
                if (!got) note_fail(err, kWaitSoftX, j);
                ok = false;
                break;
            }
            const float mt = fmaxf(mx[0], xmax[((j & 1) * 2 + (hf ^ 1)) * 64 + r]);
            float alpha = 1.f;
            bool need = false;
            if (it.seg_first()) {
                m = mt;
                lh = 0.f;
            } else if (mt > m + kRescaleThreshold) {
                alpha = ex2_approx(m - mt);
                m = mt;
                need = true;
            }
            // P = 2^(s - m) rounded to the cache type; the row sums add the fp32 values
            uint32_t pp[32];
            float sum = 0.f;
#pragma unroll
            for (int q = 0; q < 32; ++q) {
                const float e0 = ex2_approx(s[2 * q] - m), e1 = ex2_approx(s[2 * q + 1] - m);
                pp[q] = pack2<T>(e0, e1);
                sum += e0 + e1;
            }
            lh = lh * alpha + sum;
            // P slot j & 1 is free once the latent product of tile j - 2 is done
            got = j < 2 || mbar_wait_cluster(smem_u32(&bars->pv_done[j & 1]), ((j - 2) >> 1) & 1, err, code(kWaitSoftPV));
            if (!warp_ok(got)) {
                if (!got) note_fail(err, kWaitSoftPV, j);
                ok = false;
                break;
            }
            if (__any_sync(0xffffffffu, need)) {
                // the reference moved: rescale this thread's O columns (alpha = 1 elsewhere) after
                // the latent product of tile j - 1 (same group: j is not a group start here)
                got = mbar_wait_cluster(smem_u32(&bars->pv_done[(j - 1) & 1]), ((j - 1) >> 1) & 1, err, code(kWaitSoftPV));
                if (!warp_ok(got)) {
                    if (!got) note_fail(err, kWaitSoftPV, j);
                    ok = false;
                    break;
                }
                tc_fence_after();
#pragma unroll 1
                for (int c0 = 0; c0 < 256; c0 += 32) {
                    uint32_t o[32];
                    tmem_ld32_sync(tlane + kColO + c0, o);
#pragma unroll
                    for (int k = 0; k < 32; ++k) o[k] = __float_as_uint(__uint_as_float(o[k]) * alpha);
                    tmem_st32(tlane + kColO + c0, o);
                }
                tmem_st_wait();
                tc_fence_before();
            }
            {
                // P rows: chunk hf of buffer j & 1, row r, unit u at u ^ (r % 8)
                const uint32_t prow = p_u32 + (j & 1) * kPBytes + hf * kChunk + r * 128;
#pragma unroll
                for (int u = 0; u < 8; ++u)
                    asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(prow + ((u ^ (r & 7)) << 4)),
                                 "r"(pp[4 * u]), "r"(pp[4 * u + 1]), "r"(pp[4 * u + 2]), "r"(pp[4 * u + 3])
                                 : "memory");
            }
            if (np < kTile && (np & 31) != 0) {
                // the tile's straddling value chunks: zero their rows past the end
                const int kb = np >> 5, rz = np - 32 * kb;
                const int c0 = value_chunk0(j, n);
                for (int nn = 0; nn < 2; ++nn) {
                    got = mbar_wait(smem_u32(&bars->vbound[nn]), nbound & 1, err, code(kWaitBound));
                    if (!warp_ok(got)) {
                        if (!got) note_fail(err, kWaitBound, j);
                        ok = false;
                        break;
                    }
                    const int s = (c0 + 4 * nn + kb) % kNS;
                    unsigned char* ch = smem + kOffRing + s * kChunk;
                    const int units = (32 - rz) * 8;   // 16-byte units per 64-column block
                    for (int v = L; v < 2 * units; v += 128) {
                        const int blk = v / units, rem = v % units;
                        *reinterpret_cast<uint4*>(ch + blk * 4096 + (rz + rem / 8) * 128 + (rem % 8) * 16) =
                            make_uint4(0, 0, 0, 0);
                    }
                }
                if (!ok) break;
                ++nbound;
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) arrive_leader(smem_u32(&bars->p_full[j & 1]), rank);

            if (it.seg_last()) {
                // ---- group end: this worker's partial record of the group
                got = mbar_wait_cluster(smem_u32(&bars->pv_done[j & 1]), (j >> 1) & 1, err, code(kWaitSoftPV));
                if (!warp_ok(got)) {
                    if (!got) note_fail(err, kWaitSoftPV, j);
                    ok = false;
                    break;
                }
                xsum[hf * 64 + r] = lh;
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(&bars->xsum_full));
                got = mbar_wait(smem_u32(&bars->xsum_full), nsum & 1, err, code(kWaitSoftX));
                ++nsum;
                if (!warp_ok(got)) {
                    if (!got) note_fail(err, kWaitSoftX, j);
                    ok = false;
                    break;
                }
                const float l_tot = lh + xsum[(hf ^ 1) * 64 + r];
                tc_fence_after();
                const int rec = it.g + w;
                const int row = 64 * static_cast<int>(rank) + r;
                const bool row_ok = row < group_rows(P, it.g);
                float* orow = rec_o + (static_cast<long long>(rec) * kGroupRows + row) * 512 + 128 * hf;
#pragma unroll 1
                for (int nn = 0; nn < 2; ++nn) {
#pragma unroll 1
                    for (int c0 = 0; c0 < 128; c0 += 64) {
                        uint32_t o[64];
                        tmem_ld64_sync(tlane + kColO + 128 * nn + c0, o);
                        if (row_ok) {
                            st_row32(orow + 256 * nn + c0, *reinterpret_cast<const uint32_t(*)[32]>(&o[0]));
                            st_row32(orow + 256 * nn + c0 + 32, *reinterpret_cast<const uint32_t(*)[32]>(&o[32]));
                        }
                    }
                }
                if (hf == 0 && row_ok)
                    *reinterpret_cast<float2*>(rec_ml + (static_cast<long long>(rec) * kGroupRows + row) * 2) =
                        make_float2(m, l_tot);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) arrive_leader(smem_u32(&bars->o_free), rank);
            }
        }
    }

    // ---------------------------------------------------------------- teardown
    __syncthreads();
    if (threadIdx.x == 0 && *err != 0) {
        // after a failure, loads or arrivals may still be in flight towards this CTA
        const uint64_t t0 = globaltimer_ns();
        while (globaltimer_ns() - t0 < 20000ull) {
        }
    }
    tc_fence_before();
    cluster_sync();  // no CTA leaves (or frees tensor memory) while the pair may still address it
    tc_fence_after();
    if (warp == 1) tmem_dealloc_pair(tbase, kTmemCols);
}

bool decode_2sm_supported(const DecodePlan& P) {
    return P.dc == 512 && P.dR == 64 && P.tile == kTile && P.kv_rows < (1ll << 31) - 4 * kTile &&
           static_cast<long long>(P.G) * kGroupRows < (1ll << 31);
}

int decode_2sm_tile() { return kTile; }

template <typename T>
cudaError_t launch_decode_2sm(const DecodePlan& P, const T* kv, const T* qpack, const float* cos, const float* sin,
                              float* rec_ml, float* rec_o, bool pdl, cudaStream_t s) {
    if (!decode_2sm_supported(P)) return cudaErrorInvalidValue;
    Maps maps;
    const uint64_t rows = static_cast<uint64_t>(P.kv_rows), stride = static_cast<uint64_t>(P.row_stride);
    // the tables (kv_pos_offset + max_len rows of d_R / 2 = 32 floats) are read as float4
    if (!P.rope_otf && ((reinterpret_cast<uintptr_t>(cos) | reinterpret_cast<uintptr_t>(sin)) & 15u))
        return cudaErrorInvalidValue;
    if (!make_tmap_2d_16b(&maps.kv, kv, rows, 576, stride, 64, 64) ||
        !make_tmap_2d_16b(&maps.v, kv, rows, 576, stride, 32, 64) ||
        !make_tmap_2d_16b(&maps.q, qpack, static_cast<uint64_t>(P.G) * kGroupRows, 576, 576, 64, 64))
        return cudaErrorInvalidValue;
    const bool paged = P.page_table != nullptr;
    const void* kernel = paged ? reinterpret_cast<const void*>(decode_2sm_kernel<T, true>)
                               : reinterpret_cast<const void*>(decode_2sm_kernel<T, false>);
    cudaError_t e = ensure_dynamic_smem(kernel, static_cast<int>(kSmemBytes));
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * P.W);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmemBytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    if (paged)
        e = cudaLaunchKernelEx(&cfg, decode_2sm_kernel<T, true>, maps, P, cos, sin, rec_ml, rec_o);
    else
        e = cudaLaunchKernelEx(&cfg, decode_2sm_kernel<T, false>, maps, P, cos, sin, rec_ml, rec_o);
    count_launches(1);
    return e != cudaSuccess ? e : cudaGetLastError();
}

template cudaError_t launch_decode_2sm<__half>(const DecodePlan&, const __half*, const __half*, const float*,
                                               const float*, float*, float*, bool, cudaStream_t);
template cudaError_t launch_decode_2sm<__nv_bfloat16>(const DecodePlan&, const __nv_bfloat16*,
                                                      const __nv_bfloat16*, const float*, const float*, float*,
                                                      float*, bool, cudaStream_t);

}  // namespace mla
