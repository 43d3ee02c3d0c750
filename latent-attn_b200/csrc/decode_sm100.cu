// Tensor-core split-KV MLA decode for sm_100a (tcgen05 MMA, TMEM accumulators, TMA).
//
// One worker = a cluster of two CTAs (a "pair") that streams a contiguous range of
// 64-position tiles (see mla_internal.cuh for the stream-K split). All 128 query
// rows (heads) of a group form the M = 128 tile, so each cache tile is read from
// HBM once for every head.
//
// The pair splits the 576-wide score reduction and the 512-wide latent output:
//   CTA 0 owns K = c[0:256] + k_rope[0:64] (320) and output latent columns [0, 256)
//   CTA 1 owns K = c[256:512]              (256) and output latent columns [256, 512)
// so each CTA's cache slice serves both of its MMAs from the same shared memory:
//   score  S_r[128 x 64]  = Q_r(TMEM) . KV_r^T         (K-major B)
//   latent O_r[128 x 256] += P[128 x 64] . C_r[64 x 256] (P K-major, C MN-major)
// TMEM per CTA: O_r 256 columns | S 64 | Q_r 160 (CTA 0) or 128 (CTA 1).
// The full score is S_0 + S_1: each CTA rounds its partial to fp16, ships it to
// the other CTA's shared memory with st.async (completion counted on the
// receiver's mbarrier), and both add the same two fp16 halves, so both compute a
// bit-identical softmax and bit-identical P, m and l.
//
// Warp roles (256 threads):
//   warp 0      TMA producer (one lane): cache tile chunks into a 3-stage ring
//   warp 1      TMEM allocator + MMA issuer (one lane)
//   warps 2-3   tile transform: zero rows past the sequence end; CTA 0 also
//               rotates k_rope in place with the caller's fp32 cos/sin tables
//               (the rotation of src/fused_mla.cu:34-54 of the reference). The
//               producer streams each tile's 64 table rows (2 x 8 KB) with TMA into
//               a 2-slot ring next to the cache chunks, so the rotation never waits
//               on a global-memory round trip.
//   warps 4-7   softmax / correction / epilogue: thread t owns query row t
// Softmax is online in log2 units (Q is pre-scaled by softmax_scale * log2 e) with
// a lazy rescale: the running max only moves when a tile's max exceeds it by more
// than 8, which bounds P by 2^8 and makes the O rescale (TMEM ld/scale/st) rare.
// Every wait is bounded (mbar_wait*); on timeout the kernel records kStatusTimeout
// in P.status, unwinds, and the combine kernel turns the outputs into NaN.
#include <cfloat>

#include "mla_internal.cuh"
#include "sm100_ptx.cuh"
#include "tma_host.cuh"

namespace mla {
using namespace sm100;

namespace {

constexpr int kTileN = 64;                       // positions per tile
constexpr int kStages = 3;
constexpr int kChunkBytes = 64 * 128;            // 64 rows x 64 elements (128 B), 128-byte swizzle
constexpr int kStageBytes = 5 * kChunkBytes;     // CTA 0 uses 5 chunks, CTA 1 uses 4
constexpr int kTabBytes = 64 * 32 * 4;           // cos (or sin) rows of one tile, fp32
constexpr int kTabSlotBytes = 2 * kTabBytes;     // cos | sin
constexpr int kPBytes = 128 * 128;               // P: 128 rows x 64 positions x 2 B
constexpr int kXBytes = 128 * 128;               // exchanged partial score: 128 x 64 fp16
constexpr int kThreads = 256;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColO = 0, kColS = 256, kColQ = 320;
constexpr float kRescaleThreshold = 8.0f;        // log2 units

// wait-site codes recorded in the status word's upper bits (debugging aid)
enum : int { kWaitProducer = 1, kWaitTransform = 2, kWaitMmaTile = 3, kWaitMmaSFree = 4, kWaitMmaP = 5,
             kWaitMmaQ = 6, kWaitSoftS = 7, kWaitSoftX = 8, kWaitSoftPV = 9, kWaitTeardown = 10,
             kWaitDrain = 11 };

// Warp-uniform success: every early exit of a warp that runs warp-collective
// instructions (tcgen05.ld/st, vote) happens with all 32 lanes together.
__device__ __forceinline__ bool warp_ok(bool ok) { return __all_sync(0xffffffffu, ok); }

struct __align__(8) Barriers {
    uint64_t kv_full[kStages];
    uint64_t kv_empty[kStages];
    uint64_t tile_ready[kStages];
    uint64_t s_full, s_free;
    uint64_t x_full[2];
    uint64_t p_full[2];
    uint64_t pv_done[2];
    uint64_t tab_empty[2];
    uint64_t q_ready, drain, done;
    uint32_t tmem_base;
};

constexpr size_t kSmemBytes = static_cast<size_t>(kStages) * kStageBytes + 2 * kTabSlotBytes + 2 * kPBytes +
                              2 * kXBytes + sizeof(Barriers) + 1024;
static_assert(kSmemBytes <= 232448, "shared memory budget");

__device__ __forceinline__ int code(int site) { return kStatusTimeout | (site << 8); }

// Diagnostics after a wait gave up: status[1] counts failures, status[2] holds
// the first failing (block + 1) << 16 | tile, status[3] ORs the failing sites.
__device__ __forceinline__ void note_fail(volatile int* err, int site, int tile) {
    int* e = const_cast<int*>(err);
    atomicAdd(e + 1, 1);
    atomicCAS(e + 2, 0, ((static_cast<int>(blockIdx.x) + 1) << 16) | (tile & 0xFFFF));
    atomicOr(e + 3, 1 << site);
}

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
    __device__ int pos0() const { return (t - gt0) * kTileN; }
    __device__ int np() const { int r = len - pos0(); return r < kTileN ? r : kTileN; }
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

template <typename T> struct MmaFmt;
template <> struct MmaFmt<__half> { static constexpr uint32_t v = 0; };
template <> struct MmaFmt<__nv_bfloat16> { static constexpr uint32_t v = 1; };

__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}
template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float a, float b) { return pack_half2(a, b); }
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}
template <typename T>
__device__ __forceinline__ float2 unpack2(uint32_t v) {
    return ElemTraits<T>::to_f2(*reinterpret_cast<const typename ElemTraits<T>::T2*>(&v));
}

}  // namespace

template <typename T>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
decode_sm100_kernel(const __grid_constant__ CUtensorMap tmap, const __grid_constant__ CUtensorMap tmap_cos,
                    const __grid_constant__ CUtensorMap tmap_sin, const DecodePlan P, const T* __restrict__ qpack,
                    float* __restrict__ rec_ml, float* __restrict__ rec_o) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    unsigned char* stages = smem;
    unsigned char* tabs = stages + kStages * kStageBytes;
    unsigned char* pbuf = tabs + 2 * kTabSlotBytes;
    unsigned char* xbuf = pbuf + 2 * kPBytes;
    Barriers* bars = reinterpret_cast<Barriers*>(xbuf + 2 * kXBytes);

    const uint32_t rank = cluster_ctarank();
    const uint32_t peer = rank ^ 1u;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int w = blockIdx.x >> 1;
    volatile int* err = P.status;

    const int ntiles = total_tiles(P);
    if (ntiles <= 0 || w >= P.W) return;  // identical for both CTAs of the pair
    const int tb = worker_begin(ntiles, P.W, w), te = worker_begin(ntiles, P.W, w + 1);
    if (tb >= te) return;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(smem_u32(&bars->kv_full[s]), 1);
            mbar_init(smem_u32(&bars->kv_empty[s]), 1);
            mbar_init(smem_u32(&bars->tile_ready[s]), 64);
        }
        mbar_init(smem_u32(&bars->s_full), 1);
        mbar_init(smem_u32(&bars->s_free), 128);
        for (int j = 0; j < 2; ++j) {
            mbar_init(smem_u32(&bars->x_full[j]), 1);
            mbar_init(smem_u32(&bars->p_full[j]), 128);
            mbar_init(smem_u32(&bars->pv_done[j]), 1);
        }
        mbar_init(smem_u32(&bars->tab_empty[0]), 64);
        mbar_init(smem_u32(&bars->tab_empty[1]), 64);
        mbar_init(smem_u32(&bars->q_ready), 128);
        mbar_init(smem_u32(&bars->drain), 1);
        mbar_init(smem_u32(&bars->done), 1);
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(&bars->tmem_base), kTmemCols);
        tmem_relinquish();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmap);
        if (rank == 0) {
            tma_prefetch_desc(&tmap_cos);
            tma_prefetch_desc(&tmap_sin);
        }
    }
    tc_fence_before();
    cluster_sync();  // both CTAs: barriers initialised, TMEM allocated
    tc_fence_after();
    const uint32_t tbase = bars->tmem_base;

    const int nchunks = rank == 0 ? 5 : 4;
    const int ksteps = rank == 0 ? 20 : 16;   // score K / 16
    const uint32_t stages_u32 = smem_u32(stages);
    const uint32_t tabs_u32 = smem_u32(tabs);
    const uint32_t pbuf_u32 = smem_u32(pbuf);
    const uint32_t xbuf_u32 = smem_u32(xbuf);

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            TileIter it;
            it.init(P, tb, te);
            for (int i = 0; it.valid(); ++i, it.next(P)) {
                const int st = i % kStages;
                if (i >= kStages &&
                    !mbar_wait(smem_u32(&bars->kv_empty[st]), ((i / kStages) - 1) & 1, err, code(kWaitProducer))) {
                    note_fail(err, kWaitProducer, i);
                    break;
                }
                if (rank == 0 && i >= 2 &&
                    !mbar_wait(smem_u32(&bars->tab_empty[i & 1]), ((i - 2) >> 1) & 1, err, code(kWaitProducer))) {
                    note_fail(err, kWaitProducer, i);
                    break;
                }
                const uint32_t full = smem_u32(&bars->kv_full[st]);
                mbar_arrive_expect_tx(full, nchunks * kChunkBytes + (rank == 0 ? kTabSlotBytes : 0));
                const int y = static_cast<int>(it.row0 + it.pos0());
                const uint32_t dst = stages_u32 + st * kStageBytes;
                for (int j = 0; j < nchunks; ++j) {
                    const int x = rank == 0 ? (j < 4 ? 64 * j : 512) : 256 + 64 * j;
                    tma_load_2d(dst + j * kChunkBytes, &tmap, full, x, y);
                }
                if (rank == 0) {
                    const int yt = P.kv_pos_offset + it.pos0();
                    const uint32_t tdst = tabs_u32 + (i & 1) * kTabSlotBytes;
                    tma_load_2d(tdst, &tmap_cos, full, 0, yt);
                    tma_load_2d(tdst + kTabBytes, &tmap_sin, full, 0, yt);
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t fmt = MmaFmt<T>::v;
            constexpr uint32_t idesc_s = idesc_f16(128, kTileN, fmt, false, false);
            constexpr uint32_t idesc_pv = idesc_f16(128, 256, fmt, false, true);
            bool ok = true;
            auto issue_score = [&](int i) {
                const uint32_t sa = stages_u32 + (i % kStages) * kStageBytes;
                for (int k = 0; k < ksteps; ++k) {
                    const uint64_t bd = smem_desc_sw128(sa + (k >> 2) * kChunkBytes + (k & 3) * 32, 16, 1024);
                    mma_ts(tbase + kColS, tbase + kColQ + 8 * k, bd, idesc_s, k > 0 ? 1u : 0u);
                }
                mma_commit(smem_u32(&bars->s_full));
            };
            auto issue_pv = [&](int i, bool first) {
                const uint32_t sa = stages_u32 + (i % kStages) * kStageBytes;
                const uint32_t pa = pbuf_u32 + (i & 1) * kPBytes;
                for (int k = 0; k < kTileN / 16; ++k) {
                    const uint64_t ad = smem_desc_sw128(pa + 32 * k, 16, 1024);
                    const uint64_t bd = smem_desc_sw128(sa + 2048 * k, 8192, 1024);
                    mma_ss(tbase + kColO, ad, bd, idesc_pv, (first && k == 0) ? 0u : 1u);
                }
                mma_commit(smem_u32(&bars->pv_done[i & 1]));
                mma_commit(smem_u32(&bars->kv_empty[i % kStages]));
            };
            auto wait_tile = [&](int i) {
                return mbar_wait(smem_u32(&bars->tile_ready[i % kStages]), (i / kStages) & 1, err,
                                 code(kWaitMmaTile));
            };
            TileIter it;
            it.init(P, tb, te);
            int seg = 0;
            ok = mbar_wait(smem_u32(&bars->q_ready), 0, err, code(kWaitMmaQ)) && wait_tile(0);
            if (ok) {
                tc_fence_after();
                issue_score(0);
            }
            int fail_i = 0;
            for (int i = 0; ok && it.valid(); ++i) {
                fail_i = i;
                TileIter nx = it;
                nx.next(P);
                const bool has_next = nx.valid();
                const bool next_new_seg = has_next && nx.seg_first();
                if (has_next && !next_new_seg) {
                    ok = mbar_wait(smem_u32(&bars->s_free), i & 1, err, code(kWaitMmaSFree)) && wait_tile(i + 1);
                    if (!ok) break;
                    tc_fence_after();
                    issue_score(i + 1);
                }
                ok = mbar_wait(smem_u32(&bars->p_full[i & 1]), (i >> 1) & 1, err, code(kWaitMmaP));
                if (!ok) break;
                tc_fence_after();
                issue_pv(i, it.seg_first());
                if (next_new_seg) {
                    ++seg;
                    ok = mbar_wait(smem_u32(&bars->q_ready), seg & 1, err, code(kWaitMmaQ)) &&
                         mbar_wait(smem_u32(&bars->s_free), i & 1, err, code(kWaitMmaSFree)) && wait_tile(i + 1);
                    if (!ok) break;
                    tc_fence_after();
                    issue_score(i + 1);
                }
                it = nx;
            }
            if (!ok) note_fail(err, kWaitMmaP, fail_i);
            // drain: every MMA this thread issued has completed before teardown
            mma_commit(smem_u32(&bars->drain));
            mbar_wait(smem_u32(&bars->drain), 0, err, code(kWaitDrain));
        }
    } else if (warp < 4) {
        // ------------------------------------------------------------ tile transform
        const int tt = threadIdx.x - 64;  // 0..63
        TileIter it;
        it.init(P, tb, te);
        for (int i = 0; it.valid(); ++i, it.next(P)) {
            const int st = i % kStages;
            if (!mbar_wait(smem_u32(&bars->kv_full[st]), (i / kStages) & 1, err, code(kWaitTransform))) {
                note_fail(err, kWaitTransform, i);
                break;
            }
            unsigned char* sp = stages + st * kStageBytes;
            const int np = it.np();
            if (np < kTileN) {
                // zero whole rows past the sequence end (swizzle permutes within a row only)
                const int rows = kTileN - np;
                for (int v = tt; v < nchunks * rows * 8; v += 64) {
                    const int j = v / (rows * 8), rem = v % (rows * 8);
                    const int r = np + rem / 8, c = rem % 8;
                    *reinterpret_cast<uint4*>(sp + j * kChunkBytes + r * 128 + c * 16) = make_uint4(0, 0, 0, 0);
                }
            }
            if (rank == 0) {
                // rotate-half RoPE on the k_rope chunk: pairs (d, d + 32). Thread (q0, m)
                // rotates the element pairs d = 2m, 2m + 1 of rows q0, q0 + 4, ...; four rows
                // are loaded into registers before any store, so the loads of a batch
                // overlap instead of queueing behind the previous row's stores.
                unsigned char* rc = sp + 4 * kChunkBytes;
                const float* tc = reinterpret_cast<const float*>(tabs + (i & 1) * kTabSlotBytes);
                const float* ts = tc + kTabBytes / 4;
                const int m = tt & 15;
                const int q0 = tt >> 4;  // 0..3
#pragma unroll 1
                for (int pb = 0; pb < np; pb += 16) {
                    float2 cs[4], sn[4];
                    uint32_t k0[4], k1[4];
                    uint32_t* a0[4];
                    uint32_t* a1[4];
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const int p = pb + q0 + 4 * u;
                        const int sw = p & 7;
                        a0[u] = reinterpret_cast<uint32_t*>(rc + p * 128 + (((m >> 2) ^ sw) << 4) + ((m & 3) << 2));
                        a1[u] = reinterpret_cast<uint32_t*>(rc + p * 128 + ((((m >> 2) + 4) ^ sw) << 4) + ((m & 3) << 2));
                        cs[u] = *reinterpret_cast<const float2*>(tc + p * 32 + 2 * m);
                        sn[u] = *reinterpret_cast<const float2*>(ts + p * 32 + 2 * m);
                        k0[u] = *a0[u];
                        k1[u] = *a1[u];
                    }
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const int p = pb + q0 + 4 * u;
                        if (p < np) {
                            const float2 x0 = unpack2<T>(k0[u]), x1 = unpack2<T>(k1[u]);
                            *a0[u] = pack2<T>(x0.x * cs[u].x - x1.x * sn[u].x, x0.y * cs[u].y - x1.y * sn[u].y);
                            *a1[u] = pack2<T>(x0.x * sn[u].x + x1.x * cs[u].x, x0.y * sn[u].y + x1.y * cs[u].y);
                        }
                    }
                }
            }
            fence_proxy_async_smem();
            mbar_arrive(smem_u32(&bars->tile_ready[st]));
            if (rank == 0) mbar_arrive(smem_u32(&bars->tab_empty[i & 1]));
        }
    } else {
        // ------------------------------------------------------------ softmax warpgroup
        // Tile i: load S_r(i) from TMEM and release it (the score MMA of tile i+1 can
        // start), round it to fp16 and send it to the peer's X[i & 1] with st.async
        // (16 KB counted on the peer's x_full[i & 1]). Slot reuse needs no handshake:
        // the peer writes X[i & 1] again only for tile i + 2, which it reaches only
        // after receiving this CTA's tile i + 1, sent after tile i was read here.
        const int t = threadIdx.x - 128;                       // query row
        const uint32_t lane_off = static_cast<uint32_t>(32 * (warp & 3)) << 16;
        const uint32_t taddr_row = tbase + lane_off;
        const int ncol_q = rank == 0 ? 160 : 128;
        auto load_q = [&](int g) {
            const uint32_t* src = reinterpret_cast<const uint32_t*>(qpack + (static_cast<long long>(g) * 128 + t) * 576);
            for (int c = 0; c < ncol_q; c += 64) {
                uint32_t r0[32], r1[32];
                const int e0 = rank == 0 ? (c < 128 ? 2 * c : 512 + 2 * (c - 128)) : 256 + 2 * c;
                const bool two = c + 32 < ncol_q;
                const int e1 = rank == 0 ? (c + 32 < 128 ? 2 * (c + 32) : 512 + 2 * (c + 32 - 128)) : 256 + 2 * (c + 32);
                const uint4* s0 = reinterpret_cast<const uint4*>(src + e0 / 2);
                const uint4* s1 = reinterpret_cast<const uint4*>(src + e1 / 2);
#pragma unroll
                for (int v = 0; v < 8; ++v) {
                    uint4 x = __ldg(s0 + v);
                    r0[4 * v] = x.x; r0[4 * v + 1] = x.y; r0[4 * v + 2] = x.z; r0[4 * v + 3] = x.w;
                    uint4 y = two ? __ldg(s1 + v) : make_uint4(0, 0, 0, 0);
                    r1[4 * v] = y.x; r1[4 * v + 1] = y.y; r1[4 * v + 2] = y.z; r1[4 * v + 3] = y.w;
                }
                tmem_st32(taddr_row + kColQ + c, r0);
                if (two) tmem_st32(taddr_row + kColQ + c + 32, r1);
            }
            tmem_st_wait();
            tc_fence_before();
            mbar_arrive(smem_u32(&bars->q_ready));
        };

        const uint32_t x_row_local = xbuf_u32 + t * 128;
        const uint32_t x_row_remote = mapa(x_row_local, peer);
        const uint32_t p_row = pbuf_u32 + t * 128;
        const int sw = t & 7;
        TileIter it;
        it.init(P, tb, te);
        load_q(it.g);
        float m_run = 0.f, l_run = 0.f;
        for (int i = 0; it.valid(); ++i, it.next(P)) {
            const int slot = i & 1;
            if (t == 0) mbar_arrive_expect_tx(smem_u32(&bars->x_full[slot]), kXBytes);
            bool got = mbar_wait(smem_u32(&bars->s_full), i & 1, err, code(kWaitSoftS));
            if (!warp_ok(got)) {
                if (!got) note_fail(err, kWaitSoftS, i);
                break;
            }
            tc_fence_after();
            uint32_t sr[64];
            tmem_ld32(taddr_row + kColS, *reinterpret_cast<uint32_t(*)[32]>(&sr[0]));
            tmem_ld32(taddr_row + kColS + 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[32]));
            tmem_ld_wait();
            tc_fence_before();
            mbar_arrive(smem_u32(&bars->s_free));
            uint32_t h[32];
#pragma unroll
            for (int q = 0; q < 32; ++q) h[q] = pack_half2(__uint_as_float(sr[2 * q]), __uint_as_float(sr[2 * q + 1]));
            {
                const uint32_t rbar = mapa(smem_u32(&bars->x_full[slot]), peer);
                const uint32_t dst = x_row_remote + slot * kXBytes;
#pragma unroll
                for (int c = 0; c < 8; ++c)
                    st_async_v4(dst + ((c ^ sw) << 4), h[4 * c], h[4 * c + 1], h[4 * c + 2], h[4 * c + 3], rbar);
            }
            got = mbar_wait_cluster(smem_u32(&bars->x_full[slot]), (i >> 1) & 1, err, code(kWaitSoftX));
            if (!warp_ok(got)) {
                if (!got) note_fail(err, kWaitSoftX, i);
                break;
            }
            // full score = fp16(own) + fp16(peer), identical in both CTAs
            float s[64];
            const int np = it.np();
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                uint4 v;
                asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];"
                             : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                             : "r"(x_row_local + slot * kXBytes + ((c ^ sw) << 4)));
                const uint32_t pv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&h[4 * c + q]));
                    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&pv[q]));
                    const int j = 8 * c + 2 * q;
                    s[j] = j < np ? a.x + b.x : -INFINITY;
                    s[j + 1] = j + 1 < np ? a.y + b.y : -INFINITY;
                }
            }
            // tile max: tree reduction
            float mx[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) mx[j] = fmaxf(s[j], s[j + 32]);
#pragma unroll
            for (int w2 = 16; w2 > 0; w2 >>= 1)
#pragma unroll
                for (int j = 0; j < w2; ++j) mx[j] = fmaxf(mx[j], mx[j + w2]);
            const float mt = mx[0];
            float alpha = 1.f;
            bool need = false;
            if (it.seg_first()) {
                m_run = mt;
                l_run = 0.f;
            } else if (mt > m_run + kRescaleThreshold) {
                alpha = ex2_approx(m_run - mt);
                m_run = mt;
                l_run *= alpha;
                need = true;
            }
            uint32_t pp[32];
            float ls[16];
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                const uint32_t v = pack2<T>(ex2_approx(s[2 * j] - m_run), ex2_approx(s[2 * j + 1] - m_run));
                pp[j] = v;
                const float2 f = unpack2<T>(v);
                if (j < 16) ls[j] = f.x + f.y;
                else ls[j - 16] += f.x + f.y;
            }
#pragma unroll
            for (int w2 = 8; w2 > 0; w2 >>= 1)
#pragma unroll
                for (int j = 0; j < w2; ++j) ls[j] += ls[j + w2];
            l_run += ls[0];
            // P slot is free once PV(i-2) has completed
            got = i < 2 || mbar_wait(smem_u32(&bars->pv_done[slot]), ((i - 2) >> 1) & 1, err, code(kWaitSoftPV));
            if (!warp_ok(got)) {
                if (!got) note_fail(err, kWaitSoftPV, i);
                break;
            }
#pragma unroll
            for (int c = 0; c < 8; ++c)
                asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(p_row + slot * kPBytes + ((c ^ sw) << 4)),
                             "r"(pp[4 * c]), "r"(pp[4 * c + 1]), "r"(pp[4 * c + 2]), "r"(pp[4 * c + 3])
                             : "memory");
            fence_proxy_async_smem();
            if (__any_sync(0xffffffffu, need)) {
                // rescale this warp's O rows once PV(i-1) has completed
                got = mbar_wait(smem_u32(&bars->pv_done[(i - 1) & 1]), ((i - 1) >> 1) & 1, err, code(kWaitSoftPV));
                if (!warp_ok(got)) {
                    if (!got) note_fail(err, kWaitSoftPV, i);
                    break;
                }
                tc_fence_after();
#pragma unroll 1
                for (int c0 = 0; c0 < 256; c0 += 32) {
                    uint32_t o[32];
                    tmem_ld32(taddr_row + kColO + c0, o);
                    tmem_ld_wait();
#pragma unroll
                    for (int j = 0; j < 32; ++j) o[j] = __float_as_uint(__uint_as_float(o[j]) * alpha);
                    tmem_st32(taddr_row + kColO + c0, o);
                }
                tmem_st_wait();
            }
            tc_fence_before();
            mbar_arrive(smem_u32(&bars->p_full[slot]));

            if (it.seg_last()) {
                got = mbar_wait(smem_u32(&bars->pv_done[slot]), (i >> 1) & 1, err, code(kWaitSoftPV));
                if (!warp_ok(got)) {
                    if (!got) note_fail(err, kWaitSoftPV, i);
                    break;
                }
                tc_fence_after();
                const int rec = it.g + w;
                const bool row_ok = t < group_rows(P, it.g);
                float* orow = rec_o + (static_cast<long long>(rec) * kGroupRows + t) * 512 + 256 * rank;
#pragma unroll 1
                for (int c0 = 0; c0 < 256; c0 += 32) {
                    uint32_t o[32];
                    tmem_ld32(taddr_row + kColO + c0, o);
                    tmem_ld_wait();
                    if (row_ok) {
#pragma unroll
                        for (int v = 0; v < 8; ++v)
                            *reinterpret_cast<float4*>(orow + c0 + 4 * v) =
                                make_float4(__uint_as_float(o[4 * v]), __uint_as_float(o[4 * v + 1]),
                                            __uint_as_float(o[4 * v + 2]), __uint_as_float(o[4 * v + 3]));
                    }
                }
                if (rank == 0 && row_ok)
                    *reinterpret_cast<float2*>(rec_ml + (static_cast<long long>(rec) * kGroupRows + t) * 2) =
                        make_float2(m_run, l_run);
                tc_fence_before();
                if (it.t + 1 < it.t_end) {
                    TileIter nx = it;
                    nx.next(P);
                    load_q(nx.g);
                }
            }
        }
    }

    // ---------------------------------------------------------------- teardown
    __syncthreads();
    if (threadIdx.x == 0) {
        // the pair finishes together: no CTA leaves while the other may still address it
        mbar_arrive_remote(mapa(smem_u32(&bars->done), peer));
        if (!mbar_wait_cluster(smem_u32(&bars->done), 0, err, code(kWaitTeardown))) note_fail(err, kWaitTeardown, 0);
    }
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tbase, kTmemCols);
}

bool decode_sm100_available() { return true; }

template <typename T>
cudaError_t launch_decode_sm100(const DecodePlan& P, const T* kv, const T* qpack, const float* cos,
                                const float* sin, float* rec_ml, float* rec_o, cudaStream_t s) {
    if (P.dc != 512 || P.dR != 64 || P.tile != kTileN) return cudaErrorInvalidValue;
    CUtensorMap tmap, tcos, tsin;
    // tables hold kv_pos_offset + max_len rows of d_R / 2 = 32 floats
    const uint64_t trows = static_cast<uint64_t>(P.kv_pos_offset) + static_cast<uint64_t>(P.max_len);
    if (!make_tmap_2d_16b(&tmap, kv, static_cast<uint64_t>(P.kv_rows), 576, static_cast<uint64_t>(P.row_stride),
                          64, 64) ||
        !make_tmap_2d_f32(&tcos, cos, trows, 32, 32, 64, 32) || !make_tmap_2d_f32(&tsin, sin, trows, 32, 32, 64, 32))
        return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(decode_sm100_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kSmemBytes));
    if (e != cudaSuccess) return e;
    decode_sm100_kernel<T><<<2 * P.W, kThreads, kSmemBytes, s>>>(tmap, tcos, tsin, P, qpack, rec_ml, rec_o);
    count_launches(1);
    return cudaGetLastError();
}

template cudaError_t launch_decode_sm100<__half>(const DecodePlan&, const __half*, const __half*, const float*,
                                                 const float*, float*, float*, cudaStream_t);
template cudaError_t launch_decode_sm100<__nv_bfloat16>(const DecodePlan&, const __nv_bfloat16*,
                                                        const __nv_bfloat16*, const float*, const float*, float*,
                                                        float*, cudaStream_t);

}  // namespace mla
