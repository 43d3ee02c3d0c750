// Tensor-core split-KV MLA decode for sm_100a (tcgen05 MMA, TMEM accumulators, TMA).
//
// One worker = a cluster of two CTAs (a "pair") that streams a contiguous range of
// 64-position tiles (see mla_internal.cuh for the stream-K split). All 128 query
// rows (heads) of a group form the M = 128 tile, so each cache tile is read from
// HBM once for every head.
//
// The pair splits the 576-wide score reduction and the 512-wide latent output evenly:
//   CTA r owns K = c[256 r : 256 r + 256] + the 16 rotate-half frequency pairs
//   d in [16 r, 16 r + 16) of k_rope (columns d and d + 32), i.e. 288 of the 576,
//   and output latent columns [256 r, 256 r + 256).
// Each CTA's cache slice serves both of its MMAs from the same shared memory:
//   score  S_r[128 x 64]  = Q_r . KV_r^T      (16 K-steps with Q's latent part in TMEM,
//                                              2 with its rope part in shared memory)
//   latent O_r[128 x 256] += P[128 x 64](TMEM) . C_r[64 x 256]   (C read MN-major)
// TMEM per CTA: O_r 256 columns | S 64 | Q_r latent 128 | P 2 x 32.
// The full score is S_0 + S_1: each CTA rounds its partial to fp16 and ships it to
// the other CTA's shared memory with st.async (completion counted on the
// receiver's mbarrier); both add the same two fp16 halves, so both compute a
// bit-identical softmax and bit-identical P, m and l.
//
// Warp roles (384 threads):
//   warp 0      TMA producer (one lane): per tile, 4 latent chunks (128-byte swizzle) and
//               4 rope boxes of 8 columns (no swizzle), into a 5-stage ring
//   warp 1      TMEM allocator + MMA issuer (one lane): issues each tile's score (latent
//               part on arrival, rope part after the transform) and PV MMAs as soon as
//               their inputs are ready, in tile order per kind
//   warps 2-3   tile transform: zero rows past the sequence end, rotate the CTA's
//               k_rope pairs in place with the caller's cos/sin tables, read from global
//               memory one tile ahead, or with cos/sin computed on the fly (the rotation of
//               src/fused_mla.cu:34-54 of the reference)
//   warps 4-7   softmax set 0: the even tiles of the worker
//   warps 8-11  softmax set 1: the odd tiles (thread = query row = TMEM lane)
// The two softmax sets work on consecutive tiles at the same time: while one waits
// for the peer's partial scores of its tile, the other computes. Each set has its own
// P buffer in TMEM. Softmax is online in log2 units (Q is pre-scaled by
// softmax_scale * log2 e) with a lazy reference max: tile j is exponentiated against
// the reference of tile j - 1 (handed over by the other set through shared memory),
// and the reference only moves when the tile's max exceeds it by more than 8, which
// bounds P by 2^8; only then is O rescaled (rare) and the row sums re-referenced.
// Every wait is bounded (mbar_wait*); on timeout the kernel records kStatusTimeout
// in P.status, unwinds, and the merge kernel turns the outputs into NaN.
#include <cfloat>

#include "mla_internal.cuh"
#include "sm100_ptx.cuh"
#include "tma_host.cuh"

namespace mla {
using namespace sm100;

namespace {

constexpr int kTileN = 64;                          // positions per tile
constexpr int kStages = 5;
constexpr int kChunkBytes = 64 * 128;               // 64 rows x 64 latent columns, 128-byte swizzle
constexpr int kRopeBoxBytes = 64 * 16;              // 64 rows x 8 rope columns, no swizzle
constexpr int kRopeBytes = 4 * kRopeBoxBytes;
constexpr int kStageBytes = kRopeBytes + 4 * kChunkBytes;   // [rope boxes | 4 latent chunks]
constexpr int kXSlots = 2;                          // slot j & 1: its previous user is the same softmax set
constexpr int kXBytes = 128 * 128;                  // one slot: 128 rows x 64 fp16 partial scores
constexpr int kQRopeBoxBytes = 128 * 16;            // 128 rows x 8 rope elements of Q, no swizzle
constexpr int kQRopeBytes = 4 * kQRopeBoxBytes;
constexpr int kMSlots = 4;                          // reference-max hand-over slots (tile index mod 4)
constexpr int kThreads = 384;
constexpr int kTransformThreads = 64;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColO = 0, kColS = 256, kColQ = 320, kColP = 448;   // P buffers at 448 and 480
constexpr float kRescaleThreshold = 8.0f;           // log2 units

// wait-site codes recorded in the status word's upper bits (debugging aid)
enum : int { kWaitProducer = 1, kWaitTransform = 2, kWaitMma = 3, kWaitSoftS = 7, kWaitSoftX = 8,
             kWaitSoftPV = 9, kWaitTeardown = 10, kWaitDrain = 11, kWaitSoftRef = 12, kWaitCredit = 13,
             kWaitEpilogue = 14 };

// Warp-uniform success: every early exit of a warp that runs warp-collective
// instructions (tcgen05.ld/st, vote) happens with all 32 lanes together.
__device__ __forceinline__ bool warp_ok(bool ok) { return __all_sync(0xffffffffu, ok); }

struct __align__(8) Barriers {
    uint64_t kv_full[kStages];
    uint64_t kv_empty[kStages];
    uint64_t tile_ready[kStages];
    uint64_t s_full[2];               // per softmax set: score of its next tile done (score j -> s_full[j & 1])
    uint64_t s_free;
    uint64_t p_full[2], pv_done[2];   // per P buffer (tile parity)
    uint64_t x_full[kXSlots];         // the peer's partial scores of a tile arrived in this CTA
    uint64_t x_empty[kXSlots];        // credit: the peer has read what this CTA sent into that slot
    // One barrier per publication slot, not per set: a set whose tile starts a group publishes
    // without waiting for the other set, so a per-set barrier could complete two phases before
    // the other set's parity wait for the older one, which then never returns. Per slot, the next
    // phase of a slot needs the waiter's own later tiles.
    uint64_t mref[kMSlots];           // m_pub slot j % kMSlots written (tile j's reference max)
    uint64_t lpub[4];                 // l_pub slot 2 sid + ((j >> 1) & 1) written (set sid's row sum)
    uint64_t q_ready, o_free, drain, done;
    // the worker's last record: the set owning the last tile arrives once PV of that tile is done,
    // and the other set, idle by then, writes half of the record's O columns
    uint64_t epi_go;
    int epi_rec, epi_rows;            // that record's index and valid rows
    float epi_l[128];                 // and its rows' sums (an fp16 record holds o / l)
    uint32_t tmem_base;
};

constexpr size_t kSmemBytes = static_cast<size_t>(kStages) * kStageBytes +
                              static_cast<size_t>(kXSlots) * kXBytes + kQRopeBytes +
                              kMSlots * 128 * sizeof(float) + 2 * 2 * 128 * sizeof(float) + sizeof(Barriers) + 1024;
static_assert(kSmemBytes <= 232448, "shared memory budget");

__device__ __forceinline__ int code(int site) { return kStatusTimeout | (site << 8); }

// Diagnostics after a wait gave up: status[1] counts failures, status[2] holds
// the first failing (block + 1) << 16 | tile, status[3] ORs the failing sites.
static __device__ __noinline__ void note_fail(volatile int* err, int site, int tile) {
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
    // the previous tile of this worker starts a segment (so the tile before it, if any, is in another one)
    __device__ bool prev_seg_first() const { return t - 1 == t_begin || t - 1 == gt0; }
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
__device__ __forceinline__ float2 half2_to_f2(uint32_t v) {
    return __half22float2(*reinterpret_cast<const __half2*>(&v));
}

// 32 consecutive fp32 values (32-byte aligned) as four 256-bit stores.
__device__ __forceinline__ void st_row32(float* p, const uint32_t (&v)[32]) {
#pragma unroll
    for (int q = 0; q < 4; ++q)
        asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p + 8 * q), "r"(v[8 * q]),
                     "r"(v[8 * q + 1]), "r"(v[8 * q + 2]), "r"(v[8 * q + 3]), "r"(v[8 * q + 4]), "r"(v[8 * q + 5]),
                     "r"(v[8 * q + 6]), "r"(v[8 * q + 7])
                     : "memory");
}

// Writes `ncols` (a multiple of 64) columns of this thread's TMEM row to `orow` (skipped when
// !row_ok) rounded to T (o / l when RecNorm<T>, else o): 64 columns (128 bytes) at a time, as
// four 32-byte stores of this row-per-thread layout. Warp-collective.
template <typename T>
__device__ __forceinline__ void write_o_cols(uint32_t tsrc, T* orow, float inv_l, bool row_ok, int ncols) {
    for (int c0 = 0; c0 < ncols; c0 += 64) {
        uint32_t o[64];
        tmem_ld64_sync(tsrc + c0, o);
        if (row_ok) {
            uint32_t p[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                float a = __uint_as_float(o[2 * i]), b = __uint_as_float(o[2 * i + 1]);
                if constexpr (RecNorm<T>::value) {
                    a *= inv_l;
                    b *= inv_l;
                }
                p[i] = pack2<T>(a, b);
            }
            st_row32(reinterpret_cast<float*>(orow + c0), p);
        }
    }
}

// Packed two-lane fp32 arithmetic (one instruction for both lanes on sm_100).
__device__ __forceinline__ float2 f2_add(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
        "add.rn.f32x2 rd, ra, rb;\n\t"
        "mov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}
__device__ __forceinline__ float2 f2_sub(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
        "sub.rn.f32x2 rd, ra, rb;\n\t"
        "mov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}

}  // namespace

// kPaged: the cache is paged (the tile's row comes from the page table). kOtf: RoPE computed on
// the fly instead of read from the caller's tables. Separate instantiations, so each runs without
// the other modes' code: the kernel is sensitive to its instruction footprint (the page lookup
// alone cost 3.6% at B = 256).
template <typename T, bool kPaged, bool kOtf>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
decode_sm100_kernel(const __grid_constant__ CUtensorMap tmap, const __grid_constant__ CUtensorMap tmap_rope,
                    const DecodePlan P, const T* __restrict__ qpack, const float* __restrict__ cos_tab,
                    const float* __restrict__ sin_tab, float* __restrict__ rec_ml, T* __restrict__ rec_o) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    unsigned char* stages = smem;
    unsigned char* xbuf = stages + kStages * kStageBytes;
    unsigned char* qrope = xbuf + kXSlots * kXBytes;                       // Q's rope part, 4 core-matrix boxes
    float* m_pub = reinterpret_cast<float*>(qrope + kQRopeBytes);         // [kMSlots][128]: reference max of tile j
    float* l_pub = m_pub + kMSlots * 128;  // [set][2][128]: row sum over the set's tiles, referenced to m_pub of its latest
    Barriers* bars = reinterpret_cast<Barriers*>(l_pub + 2 * 2 * 128);

    const uint32_t rank = cluster_ctarank();
    const uint32_t peer = rank ^ 1u;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int w = blockIdx.x >> 1;
    volatile int* err = P.status;

    if (threadIdx.x == 0) {
        pdl_launch_dependents();
        // the first TMA of each map waits for its descriptor: fetch both right away
        tma_prefetch_desc(&tmap);
        tma_prefetch_desc(&tmap_rope);
    }
    // With variable lengths the tile prefix comes from the query-packing kernel: wait for it
    // before walking tiles. With uniform lengths only the packed queries depend on that
    // kernel, and only the softmax warps read them.
    const bool uniform = P.uniform_len > 0;
    if (!uniform) pdl_wait();
    const int ntiles = total_tiles(P);
    if (ntiles <= 0 || w >= P.W) return;  // identical for both CTAs of the pair
    const int tb = worker_begin(ntiles, P.W, w), te = worker_begin(ntiles, P.W, w + 1);
    if (tb >= te) return;
    const int n = te - tb;  // tiles of this worker

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(smem_u32(&bars->kv_full[s]), 1);
            mbar_init(smem_u32(&bars->kv_empty[s]), 1);
            mbar_init(smem_u32(&bars->tile_ready[s]), kTransformThreads);
        }
        mbar_init(smem_u32(&bars->s_full[0]), 1);
        mbar_init(smem_u32(&bars->s_full[1]), 1);
        mbar_init(smem_u32(&bars->s_free), 128);
        for (int b = 0; b < 2; ++b) {
            mbar_init(smem_u32(&bars->p_full[b]), 128);
            mbar_init(smem_u32(&bars->pv_done[b]), 1);
        }
        for (int b = 0; b < kMSlots; ++b) mbar_init(smem_u32(&bars->mref[b]), 128);
        for (int b = 0; b < 4; ++b) mbar_init(smem_u32(&bars->lpub[b]), 128);
        for (int s = 0; s < kXSlots; ++s) {
            mbar_init(smem_u32(&bars->x_full[s]), 1);
            mbar_init(smem_u32(&bars->x_empty[s]), 4);  // one arrival per warp of the peer's reading set
        }
        mbar_init(smem_u32(&bars->q_ready), 128);
        mbar_init(smem_u32(&bars->o_free), 128);
        mbar_init(smem_u32(&bars->drain), 1);
        mbar_init(smem_u32(&bars->done), 1);
        mbar_init(smem_u32(&bars->epi_go), 128);
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(&bars->tmem_base), kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    cluster_sync();  // both CTAs: barriers initialised, TMEM allocated
    tc_fence_after();
    const uint32_t tbase = bars->tmem_base;
    const uint32_t stages_u32 = smem_u32(stages);
    const uint32_t xbuf_u32 = smem_u32(xbuf);
    const uint32_t qrope_u32 = smem_u32(qrope);

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            // a paged producer may record kStatusBadPage: the previous kernel clears the status
            // words, so wait for it first (with variable lengths every role waited already)
            if constexpr (kPaged)
                if (uniform) pdl_wait();
            TileIter it;
            it.init(P, tb, te);
            int issued = 0;
            for (int i = 0; it.valid(); ++i, it.next(P)) {
                const int st = i % kStages;
                // paged: the tile's cache row from the page table, read before the stage wait so its
                // latency overlaps it
                long long kvr = 0;
                if constexpr (kPaged) kvr = tile_kv_row(P, it.g, it.row0, it.pos0());
                if (i >= kStages &&
                    !mbar_wait(smem_u32(&bars->kv_empty[st]), ((i / kStages) - 1) & 1, err, code(kWaitProducer))) {
                    note_fail(err, kWaitProducer, i);
                    break;
                }
                const uint32_t full = smem_u32(&bars->kv_full[st]);
                mbar_arrive_expect_tx(full, kStageBytes);
                int y = static_cast<int>(it.row0 + it.pos0());
                if constexpr (kPaged) {
                    // a page outside the cache: the loads start below row 0 and read zeros
                    if (kvr < 0) atomicCAS(const_cast<int*>(err), 0, kStatusBadPage);
                    y = kvr < 0 ? -2 * kTileN : static_cast<int>(kvr);
                }
                const uint32_t dst = stages_u32 + st * kStageBytes;
                // rope boxes: columns 16 r + {0, 8} and 32 + 16 r + {0, 8} of k_rope
                for (int b = 0; b < 4; ++b)
                    tma_load_2d(dst + b * kRopeBoxBytes, &tmap_rope, full,
                                P.dc + 16 * static_cast<int>(rank) + 8 * (b & 1) + 32 * (b >> 1), y);
                for (int j = 0; j < 4; ++j)
                    tma_load_2d(dst + kRopeBytes + j * kChunkBytes, &tmap, full, 256 * static_cast<int>(rank) + 64 * j, y);
                issued = i + 1;
            }
            // shared memory must not be released under a TMA write: the last kStages loads (the
            // earlier ones were consumed before their stage was refilled) land before teardown,
            // also when another role gave up early
            for (int i = issued > kStages ? issued - kStages : 0; i < issued; ++i)
                mbar_wait(smem_u32(&bars->kv_full[i % kStages]), (i / kStages) & 1, err, code(kWaitProducer), 100000000ull);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t fmt = MmaFmt<T>::v;
            constexpr uint32_t idesc_s = idesc_f16(128, kTileN, fmt, false, false);
            constexpr uint32_t idesc_pv = idesc_f16(128, 256, fmt, false, true);
            // The issue loops are fully unrolled over precomputed descriptors: adding (bytes >> 4)
            // to a descriptor advances its 14-bit start-address field (shared addresses stay
            // below 2^18, so the field never carries).
            const uint32_t tS = tbase + kColS, tQ = tbase + kColQ, tO = tbase + kColO;
            const uint64_t dqr = smem_desc_noswz(qrope_u32, kQRopeBoxBytes, 128);   // Q rope, A operand
            // The latent part of a score reads only the landed stage and Q, so it is issued as soon
            // as the stage lands and runs while the transform rotates the rope part (rows past a
            // sequence end may still be zeroed meanwhile: their score columns are masked).
            auto issue_score_latent = [&](int i) {
                const uint32_t sa = stages_u32 + (i % kStages) * kStageBytes;
                const uint64_t dl = smem_desc_sw128(sa + kRopeBytes, 16, 1024);
                mma_ts(tS, tQ, dl, idesc_s, 0u);
#pragma unroll
                for (int k = 1; k < 16; ++k)
                    mma_ts(tS, tQ + 8 * k, dl + static_cast<uint64_t>(((k >> 2) * kChunkBytes + (k & 3) * 32) >> 4),
                           idesc_s, 1u);
            };
            auto issue_score_rope = [&](int i) {
                const uint32_t sa = stages_u32 + (i % kStages) * kStageBytes;
                const uint64_t dr = smem_desc_noswz(sa, kRopeBoxBytes, 128);
                // rope: two 8-column core-matrix boxes per K = 16 step, 8-row groups 128 bytes apart
                mma_ss(tS, dqr, dr, idesc_s, 1u);
                mma_ss(tS, dqr + static_cast<uint64_t>((2 * kQRopeBoxBytes) >> 4),
                       dr + static_cast<uint64_t>((2 * kRopeBoxBytes) >> 4), idesc_s, 1u);
                mma_commit(smem_u32(&bars->s_full[i & 1]));
            };
            auto issue_pv = [&](int i, bool first) {
                const uint64_t dc = smem_desc_sw128(stages_u32 + (i % kStages) * kStageBytes + kRopeBytes, 8192, 1024);
                const uint32_t tP = tbase + kColP + 32 * (i & 1);
                mma_ts(tO, tP, dc, idesc_pv, first ? 0u : 1u);
#pragma unroll
                for (int k = 1; k < kTileN / 16; ++k)
                    mma_ts(tO, tP + 8 * k, dc + static_cast<uint64_t>((2048 * k) >> 4), idesc_pv, 1u);
                mma_commit(smem_u32(&bars->pv_done[i & 1]));
                mma_commit(smem_u32(&bars->kv_empty[i % kStages]));
            };
            // Scores and PVs are each issued in tile order, but interleaved as their inputs
            // become ready: the latent part of score(s) needs S released (s_free of tile s - 1),
            // its stage landed and, at a group start, the group's Q; the rope part needs the stage
            // transformed; PV(v) needs P(v) and, at a group start after the first, the previous
            // group's O read out (o_free).
            TileIter its, itv;
            its.init(P, tb, te);
            itv = its;
            int next_s = 0, next_r = 0, next_v = 0, qseg = 0, vseg = 0;
            bool ok = true;
            long long t_last = clock64();
            const long long budget = wait_budget_cycles(kDefaultWaitNs);
            for (uint32_t spin = 0; ok && next_v < n; ++spin) {
                bool progressed = false;
                if (next_s < n && next_r == next_s) {
                    bool ready = (next_s == 0 || mbar_test(smem_u32(&bars->s_free), (next_s - 1) & 1)) &&
                                 mbar_test(smem_u32(&bars->kv_full[next_s % kStages]), (next_s / kStages) & 1) &&
                                 (!its.seg_first() || mbar_test(smem_u32(&bars->q_ready), qseg & 1));
                    if (ready) {
                        tc_fence_after();
                        issue_score_latent(next_s);
                        if (its.seg_last()) ++qseg;
                        its.next(P);
                        ++next_s;
                        progressed = true;
                    }
                }
                if (next_r < next_s &&
                    mbar_test(smem_u32(&bars->tile_ready[next_r % kStages]), (next_r / kStages) & 1)) {
                    tc_fence_after();
                    issue_score_rope(next_r);
                    ++next_r;
                    progressed = true;
                }
                if (next_v < next_r) {
                    bool ready = mbar_test(smem_u32(&bars->p_full[next_v & 1]), (next_v >> 1) & 1) &&
                                 (!itv.seg_first() || vseg == 0 || mbar_test(smem_u32(&bars->o_free), (vseg - 1) & 1));
                    if (ready) {
                        tc_fence_after();
                        issue_pv(next_v, itv.seg_first());
                        if (itv.seg_last()) ++vseg;
                        itv.next(P);
                        ++next_v;
                        progressed = true;
                    }
                }
                if (progressed) {
                    t_last = clock64();
                    continue;
                }
                // no back-off between polls: a sleep delays the next issue by more than the
                // issue slots the polls take from the softmax warps (about 1.5% of the kernel time)
                if ((spin & 31u) == 0u) {
                    const long long dt = clock64() - t_last;
                    if ((dt > kErrPollCycles && *err != 0) || dt > budget) {
                        atomicCAS(const_cast<int*>(err), 0, code(kWaitMma));
                        note_fail(err, kWaitMma, next_v);
                        ok = false;
                    }
                }
            }
            // drain: every MMA this thread issued has completed before teardown
            mma_commit(smem_u32(&bars->drain));
            mbar_wait(smem_u32(&bars->drain), 0, err, code(kWaitDrain));
        }
    } else if (warp < 4) {
        // ------------------------------------------------------------ tile transform
        const int tt = threadIdx.x - 64;  // 0 .. kTransformThreads - 1
        // rotate-half RoPE of this CTA's 16 frequency pairs: item (row p, half h) rotates
        // box h (columns 16 r + 8 h ..) against box 2 + h (columns 32 + 16 r + 8 h ..) with the
        // 8 cos / sin values of table row kv_pos_offset + position, columns 16 r + 8 h ..
        // Each thread owns items tt and tt + 64 of every tile and reads their table values
        // from global memory one tile ahead, so the loads overlap the tile before.
        constexpr int kItems = 128 / kTransformThreads;
        float4 tab_next[kItems][4];  // per item: cos[0:4], cos[4:8], sin[0:4], sin[4:8]
        // Both items of a thread have the same half h = tt & 1, i.e. the same 8 frequencies.
        // On-the-fly RoPE: the angle (P0 + p) f of the tile's base position P0 and the item's
        // offset p is rotated as base(P0 f) x step(p f): the 16 base rotations of a tile are
        // computed by lanes 0-15 and shuffled; each thread's 2 x 8 step rotations once per CTA.
        const int hsel = tt & 1;
        const int f0 = 16 * static_cast<int>(rank) + 8 * hsel;
        float stc[kItems][8], sts[kItems][8];
        if constexpr (kOtf) {
#pragma unroll
            for (int u = 0; u < kItems; ++u)
#pragma unroll
                for (int e = 0; e < 8; ++e)
                    rope_sincos_exact((tt + kTransformThreads * u) >> 1, P.rope_freq[f0 + e], &sts[u][e], &stc[u][e]);
        }
        auto load_tabs = [&](const TileIter& ti) {
            const int tnp = ti.np();
            const long long pos0 = static_cast<long long>(P.kv_pos_offset) + ti.pos0();
            if constexpr (kOtf) {
                // computed, not read: no table traffic and no load latency (warp-collective)
                float cb = 1.f, sb = 0.f;
                if (lane < 16) rope_sincos_exact(pos0, P.rope_freq[16 * static_cast<int>(rank) + lane], &sb, &cb);
                float cs[kItems][8], sn[kItems][8];
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const float c0 = __shfl_sync(0xffffffffu, cb, 8 * hsel + e);
                    const float s0 = __shfl_sync(0xffffffffu, sb, 8 * hsel + e);
#pragma unroll
                    for (int u = 0; u < kItems; ++u) {
                        cs[u][e] = c0 * stc[u][e] - s0 * sts[u][e];
                        sn[u][e] = s0 * stc[u][e] + c0 * sts[u][e];
                    }
                }
#pragma unroll
                for (int u = 0; u < kItems; ++u) {
                    tab_next[u][0] = make_float4(cs[u][0], cs[u][1], cs[u][2], cs[u][3]);
                    tab_next[u][1] = make_float4(cs[u][4], cs[u][5], cs[u][6], cs[u][7]);
                    tab_next[u][2] = make_float4(sn[u][0], sn[u][1], sn[u][2], sn[u][3]);
                    tab_next[u][3] = make_float4(sn[u][4], sn[u][5], sn[u][6], sn[u][7]);
                }
            } else {
#pragma unroll
            for (int u = 0; u < kItems; ++u) {
                const int item = tt + kTransformThreads * u, p = item >> 1;
                if (p < tnp) {
                    const long long off = (pos0 + p) * 32 + f0;
                    const float4* c4 = reinterpret_cast<const float4*>(cos_tab + off);
                    const float4* s4 = reinterpret_cast<const float4*>(sin_tab + off);
                    tab_next[u][0] = __ldg(c4);
                    tab_next[u][1] = __ldg(c4 + 1);
                    tab_next[u][2] = __ldg(s4);
                    tab_next[u][3] = __ldg(s4 + 1);
                }
            }
            }
        };
        TileIter it;
        it.init(P, tb, te);
        load_tabs(it);
        for (int i = 0; it.valid(); ++i, it.next(P)) {
            const int st = i % kStages;
            float4 tab[kItems][4];
#pragma unroll
            for (int u = 0; u < kItems; ++u)
#pragma unroll
                for (int q = 0; q < 4; ++q) tab[u][q] = tab_next[u][q];
            {
                TileIter nx = it;
                nx.next(P);
                if (nx.valid()) load_tabs(nx);
            }
            if (!mbar_wait(smem_u32(&bars->kv_full[st]), (i / kStages) & 1, err, code(kWaitTransform))) {
                note_fail(err, kWaitTransform, i);
                break;
            }
            unsigned char* sp = stages + st * kStageBytes;
            const int np = it.np();
            if (np < kTileN) {
                // zero whole rows past the sequence end (swizzle permutes within a row only)
                const int rows = kTileN - np;
                for (int v = tt; v < 4 * rows * 8; v += kTransformThreads) {
                    const int j = v / (rows * 8), rem = v % (rows * 8);
                    const int r = np + rem / 8, c = rem % 8;
                    *reinterpret_cast<uint4*>(sp + kRopeBytes + j * kChunkBytes + r * 128 + c * 16) =
                        make_uint4(0, 0, 0, 0);
                }
                for (int v = tt; v < 4 * rows; v += kTransformThreads)
                    *reinterpret_cast<uint4*>(sp + (v / rows) * kRopeBoxBytes + (np + v % rows) * 16) =
                        make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int u = 0; u < kItems; ++u) {
                const int item = tt + kTransformThreads * u, p = item >> 1, h = item & 1;
                if (p < np) {
                    uint4* a = reinterpret_cast<uint4*>(sp + h * kRopeBoxBytes + p * 16);
                    uint4* b = reinterpret_cast<uint4*>(sp + (2 + h) * kRopeBoxBytes + p * 16);
                    const uint4 ka = *a, kb = *b;
                    const float cs[8] = {tab[u][0].x, tab[u][0].y, tab[u][0].z, tab[u][0].w,
                                         tab[u][1].x, tab[u][1].y, tab[u][1].z, tab[u][1].w};
                    const float sn[8] = {tab[u][2].x, tab[u][2].y, tab[u][2].z, tab[u][2].w,
                                         tab[u][3].x, tab[u][3].y, tab[u][3].z, tab[u][3].w};
                    const uint32_t xa[4] = {ka.x, ka.y, ka.z, ka.w}, xb[4] = {kb.x, kb.y, kb.z, kb.w};
                    uint32_t ya[4], yb[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float2 x0 = unpack2<T>(xa[e]), x1 = unpack2<T>(xb[e]);
                        const float c_lo = cs[2 * e], c_hi = cs[2 * e + 1], s_lo = sn[2 * e], s_hi = sn[2 * e + 1];
                        ya[e] = pack2<T>(x0.x * c_lo - x1.x * s_lo, x0.y * c_hi - x1.y * s_hi);
                        yb[e] = pack2<T>(x0.x * s_lo + x1.x * c_lo, x0.y * s_hi + x1.y * c_hi);
                    }
                    *a = make_uint4(ya[0], ya[1], ya[2], ya[3]);
                    *b = make_uint4(yb[0], yb[1], yb[2], yb[3]);
                }
            }
            fence_proxy_async_smem();
            mbar_arrive(smem_u32(&bars->tile_ready[st]));
        }
    } else {
        // ------------------------------------------------------------ softmax sets
        const int sid = (warp - 4) >> 2;                        // set: tiles j with j % 2 == sid
        const int t = (warp & 3) * 32 + lane;                   // query row == TMEM lane
        const uint32_t trow = tbase + (static_cast<uint32_t>(32 * (warp & 3)) << 16);
        // exchange layout: 16-byte chunk c of row t at c * 2048 + t * 16, so each warp-wide
        // st.async / ld.shared covers 512 contiguous bytes
        const uint32_t x_local = xbuf_u32 + t * 16;
        const uint32_t x_remote = mapa(x_local, peer);
        if (uniform) pdl_wait();  // packed queries come from the previous kernel

        // Q of group g: latent part (K elements 256 r .. 256 r + 256) into TMEM columns
        // [kColQ, kColQ + 128), two elements per column; rope part (rope 16 r .. 16 r + 16 and
        // 32 + 16 r .. + 16) into the 4 core-matrix boxes of qrope. Loaded in two halves so at
        // most 20 16-byte values are in flight per thread.
        auto load_q = [&](int g) {
            const T* src = qpack + (static_cast<long long>(g) * kGroupRows + t) * (P.dc + P.dR);
            const uint4* lat = reinterpret_cast<const uint4*>(src + 256 * rank);
            {
                uint4 v[16], r[4];
#pragma unroll
                for (int k = 0; k < 16; ++k) v[k] = __ldg(lat + k);
                const uint4* r0 = reinterpret_cast<const uint4*>(src + P.dc + 16 * rank);
                const uint4* r1 = reinterpret_cast<const uint4*>(src + P.dc + 32 + 16 * rank);
                r[0] = __ldg(r0);
                r[1] = __ldg(r0 + 1);
                r[2] = __ldg(r1);
                r[3] = __ldg(r1 + 1);
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const uint32_t x[16] = {v[4 * q].x, v[4 * q].y, v[4 * q].z, v[4 * q].w,
                                            v[4 * q + 1].x, v[4 * q + 1].y, v[4 * q + 1].z, v[4 * q + 1].w,
                                            v[4 * q + 2].x, v[4 * q + 2].y, v[4 * q + 2].z, v[4 * q + 2].w,
                                            v[4 * q + 3].x, v[4 * q + 3].y, v[4 * q + 3].z, v[4 * q + 3].w};
                    tmem_st16(trow + kColQ + 16 * q, x);
                }
#pragma unroll
                for (int b = 0; b < 4; ++b)
                    *reinterpret_cast<uint4*>(qrope + b * kQRopeBoxBytes + t * 16) = r[b];
            }
            {
                uint4 v[16];
#pragma unroll
                for (int k = 0; k < 16; ++k) v[k] = __ldg(lat + 16 + k);
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const uint32_t x[16] = {v[4 * q].x, v[4 * q].y, v[4 * q].z, v[4 * q].w,
                                            v[4 * q + 1].x, v[4 * q + 1].y, v[4 * q + 1].z, v[4 * q + 1].w,
                                            v[4 * q + 2].x, v[4 * q + 2].y, v[4 * q + 2].z, v[4 * q + 2].w,
                                            v[4 * q + 3].x, v[4 * q + 3].y, v[4 * q + 3].z, v[4 * q + 3].w};
                    tmem_st16(trow + kColQ + 64 + 16 * q, x);
                }
            }
            fence_proxy_async_smem();
            tmem_st_wait();
            tc_fence_before();
            mbar_arrive(smem_u32(&bars->q_ready));
        };

        TileIter it;
        it.init(P, tb, te);
        if (sid == 1) it.next(P);
        else load_q(it.g);        // the first tile (a group start) belongs to set 0
        float l_self = 0.f, m_l = 0.f;   // this set's row sum over its tiles of the group, and its reference
        bool ok = true;
        for (int j = sid; ok && it.valid(); j += 2) {
            const int slot = j % kXSlots;
            // ---- phase A: S_r(j) -> registers, release S, next group's Q, send the fp16 partial.
            // Every barrier below is waited on phase by phase by its waiters: a parity wait must
            // never start while the barrier is still one phase short (it would pass at once).
            // s_full[sid] holds only this set's tiles for that reason.
            bool got = mbar_wait(smem_u32(&bars->s_full[sid]), (j >> 1) & 1, err, code(kWaitSoftS));
            if (!warp_ok(got)) {
                if (!got) note_fail(err, kWaitSoftS, j);
                break;
            }
            // the slot's previous user is this set's tile j - 2, whose data this set has already
            // waited for: the slot's previous phase is complete before this arrival opens the next
            if (t == 0) mbar_arrive_expect_tx(smem_u32(&bars->x_full[slot]), kXBytes);
            tc_fence_after();
            uint32_t h[32];
            {
                uint32_t sr[64];
                tmem_ld64_sync(trow + kColS, sr);
                tc_fence_before();
                mbar_arrive(smem_u32(&bars->s_free));
#pragma unroll
                for (int q = 0; q < 32; ++q) h[q] = pack_half2(__uint_as_float(sr[2 * q]), __uint_as_float(sr[2 * q + 1]));
            }
            if (it.seg_last() && it.t + 1 < it.t_end) {
                // the score of tile j was the last MMA to read this group's Q
                TileIter nx = it;
                nx.next(P);
                load_q(nx.g);
            }
            // the peer reads its slot for tile j - 2 before this CTA writes it again
            got = j < kXSlots ||
                  mbar_wait_cluster(smem_u32(&bars->x_empty[slot]), ((j / kXSlots) - 1) & 1, err, code(kWaitCredit));
            if (!warp_ok(got)) {
                if (!got) note_fail(err, kWaitCredit, j);
                break;
            }
            {
                const uint32_t rbar = mapa(smem_u32(&bars->x_full[slot]), peer);
                const uint32_t dst = x_remote + slot * kXBytes;
#pragma unroll
                for (int c = 0; c < 8; ++c)
                    st_async_v4(dst + c * 2048, h[4 * c], h[4 * c + 1], h[4 * c + 2], h[4 * c + 3], rbar);
            }

            // ---- phase B: full score, reference max, P into TMEM buffer j & 1
            got = mbar_wait_cluster(smem_u32(&bars->x_full[slot]), (j / kXSlots) & 1, err, code(kWaitSoftX));
            if (!warp_ok(got)) {
                if (!got) note_fail(err, kWaitSoftX, j);
                break;
            }
            float s[64];
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                uint4 v;
                asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];"
                             : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                             : "r"(x_local + slot * kXBytes + c * 2048));
                const uint32_t pv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float2 r = f2_add(half2_to_f2(h[4 * c + q]), half2_to_f2(pv[q]));
                    s[8 * c + 2 * q] = r.x;
                    s[8 * c + 2 * q + 1] = r.y;
                }
            }
            // credit for the peer: this warp's rows of the slot are read. The arrive is relaxed: a
            // cluster-scope release would first wait for the acknowledgement of this thread's
            // st.async stores above (most of a microsecond under load). What it must follow are
            // reads of this CTA's own shared memory, issued before the __syncwarp; the peer writes
            // the slot again only after this arrive has crossed the cluster and the peer has
            // observed it and sent new data back.
            __syncwarp();
            if (lane == 0) mbar_arrive_remote_relaxed(mapa(smem_u32(&bars->x_empty[slot]), peer));
            const int np = it.np();
            if (np < kTileN) {
                // the group's last tile: positions past the sequence end take no weight
#pragma unroll
                for (int k = 0; k < kTileN; ++k)
                    if (k >= np) s[k] = -INFINITY;
            }
            float mx[32];
#pragma unroll
            for (int k = 0; k < 32; ++k) mx[k] = fmaxf(s[k], s[k + 32]);
#pragma unroll
            for (int w2 = 16; w2 > 0; w2 >>= 1)
#pragma unroll
                for (int k = 0; k < w2; ++k) mx[k] = fmaxf(mx[k], mx[k + w2]);
            const float mt = mx[0];
            // reference max: the previous tile's (from the other set) unless this tile exceeds it by
            // more than the threshold
            float m = mt, alpha = 1.f;
            bool need = false;
            if (!it.seg_first()) {
                got = mbar_wait(smem_u32(&bars->mref[(j - 1) % kMSlots]), ((j - 1) / kMSlots) & 1, err, code(kWaitSoftRef));
                if (!warp_ok(got)) {
                    if (!got) note_fail(err, kWaitSoftRef, j);
                    break;
                }
                const float m_prev = m_pub[((j - 1) % kMSlots) * 128 + t];
                if (mt > m_prev + kRescaleThreshold) {
                    alpha = ex2_approx(m_prev - mt);
                    need = true;
                } else {
                    m = m_prev;
                }
            }
            m_pub[(j % kMSlots) * 128 + t] = m;
            mbar_arrive(smem_u32(&bars->mref[j % kMSlots]));
            // P = 2^(s - m) rounded to the cache type for the PV MMA; the row sum adds the fp32 values
            uint32_t pp[32];
            float2 ls[8];
            const float2 m2 = make_float2(m, m);
#pragma unroll
            for (int q = 0; q < 32; ++q) {
                const float2 d = f2_sub(make_float2(s[2 * q], s[2 * q + 1]), m2);
                const float2 e = make_float2(ex2_approx(d.x), ex2_approx(d.y));
                pp[q] = pack2<T>(e.x, e.y);
                ls[q & 7] = q < 8 ? e : f2_add(ls[q & 7], e);
            }
#pragma unroll
            for (int w2 = 4; w2 > 0; w2 >>= 1)
#pragma unroll
                for (int k = 0; k < w2; ++k) ls[k] = f2_add(ls[k], ls[k + w2]);
            // this set's row sum restarts at its first tile of a group and follows the reference
            if (it.seg_first() || it.prev_seg_first()) {
                l_self = 0.f;
            } else if (m != m_l) {
                l_self *= ex2_approx(m_l - m);
            }
            m_l = m;
            l_self += ls[0].x + ls[0].y;
            // P buffer j & 1 is free once PV(j - 2) has completed
            got = j < 2 || mbar_wait(smem_u32(&bars->pv_done[j & 1]), ((j - 2) >> 1) & 1, err, code(kWaitSoftPV));
            if (!warp_ok(got)) {
                if (!got) note_fail(err, kWaitSoftPV, j);
                break;
            }
            if (__any_sync(0xffffffffu, need)) {
                // the reference moved: rescale O (alpha = 1 on rows that keep theirs) once PV(j - 1) is done
                got = mbar_wait(smem_u32(&bars->pv_done[(j - 1) & 1]), ((j - 1) >> 1) & 1, err, code(kWaitSoftPV));
                if (!warp_ok(got)) {
                    if (!got) note_fail(err, kWaitSoftPV, j);
                    break;
                }
                tc_fence_after();
#pragma unroll 1
                for (int c0 = 0; c0 < 256; c0 += 32) {
                    uint32_t o[32];
                    tmem_ld32_sync(trow + kColO + c0, o);
#pragma unroll
                    for (int k = 0; k < 32; ++k) o[k] = __float_as_uint(__uint_as_float(o[k]) * alpha);
                    tmem_st32(trow + kColO + c0, o);
                }
            }
            tc_fence_after();
            tmem_st32(trow + kColP + 32 * (j & 1), pp);
            tmem_st_wait();
            tc_fence_before();
            mbar_arrive(smem_u32(&bars->p_full[j & 1]));
            // publish this set's row sum (slot by the set's tile count)
            l_pub[(sid * 2 + ((j >> 1) & 1)) * 128 + t] = l_self;
            mbar_arrive(smem_u32(&bars->lpub[sid * 2 + ((j >> 1) & 1)]));

            if (it.seg_last()) {
                // ---- group end: partial record of this worker
                got = mbar_wait(smem_u32(&bars->pv_done[j & 1]), (j >> 1) & 1, err, code(kWaitSoftPV));
                int site = kWaitSoftPV;
                float l_tot = l_self;
                if (warp_ok(got) && !it.seg_first()) {
                    site = kWaitSoftRef;
                    // the other set's tiles of the group end at tile j - 1
                    got = mbar_wait(smem_u32(&bars->lpub[(sid ^ 1) * 2 + (((j - 1) >> 1) & 1)]), ((j - 1) >> 2) & 1, err,
                                   code(kWaitSoftRef));
                    // its reference is tile j - 1's, still in m_pub (tile j + 3 overwrites that slot)
                    const float lo = l_pub[((sid ^ 1) * 2 + (((j - 1) >> 1) & 1)) * 128 + t];
                    l_tot += lo * ex2_approx(m_pub[((j - 1) % kMSlots) * 128 + t] - m);
                }
                if (!warp_ok(got)) {
                    if (!got) note_fail(err, site, j);
                    break;
                }
                tc_fence_after();
                const int rec = it.g + w;
                const int rows = group_rows(P, it.g);
                // the worker's last tile: the other set has no tile left and writes columns 128..255
                const bool shared_epi = j == n - 1;
                if (shared_epi) {
                    if (t == 0) {
                        bars->epi_rec = rec;
                        bars->epi_rows = rows;
                    }
                    bars->epi_l[t] = l_tot;
                    tc_fence_before();
                    mbar_arrive(smem_u32(&bars->epi_go));
                }
                write_o_cols<T>(trow + kColO, rec_o + (static_cast<long long>(rec) * kGroupRows + t) * 512 + 256 * rank,
                                l_tot > 0.f ? 1.f / l_tot : 0.f, t < rows, shared_epi ? 128 : 256);
                if (rank == 0 && t < rows)
                    *reinterpret_cast<float2*>(rec_ml + (static_cast<long long>(rec) * kGroupRows + t) * 2) =
                        make_float2(m, l_tot);
                tc_fence_before();
                mbar_arrive(smem_u32(&bars->o_free));
            }
            it.next(P);
            it.next(P);
        }
        if (ok && ((n - 1) & 1) != sid) {
            // the worker's last tile is the other set's: write columns 128..255 of its record
            const bool got = mbar_wait(smem_u32(&bars->epi_go), 0, err, code(kWaitEpilogue));
            if (warp_ok(got)) {
                tc_fence_after();
                const int rec = bars->epi_rec;
                const float le = bars->epi_l[t];
                write_o_cols<T>(trow + kColO + 128,
                                rec_o + (static_cast<long long>(rec) * kGroupRows + t) * 512 + 256 * rank + 128,
                                le > 0.f ? 1.f / le : 0.f, t < bars->epi_rows, 128);
            } else if (!got) {
                note_fail(err, kWaitEpilogue, n - 1);
            }
        }
    }

    // ---------------------------------------------------------------- teardown
    __syncthreads();
    if (threadIdx.x == 0) {
        // the pair finishes together: no CTA leaves while the other may still address it
        mbar_arrive_remote(mapa(smem_u32(&bars->done), peer));
        if (!mbar_wait_cluster_full(smem_u32(&bars->done), 0, err, code(kWaitTeardown)))
            note_fail(err, kWaitTeardown, 0);
    }
    if (threadIdx.x == 0 && *err != 0) {
        // after a failure the peer may still have partial scores in flight towards this CTA
        const uint64_t t0 = globaltimer_ns();
        while (globaltimer_ns() - t0 < 20000ull) {
        }
    }
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tbase, kTmemCols);
}

bool decode_sm100_available() { return true; }

template <typename T>
cudaError_t launch_decode_sm100(const DecodePlan& P, const T* kv, const T* qpack, const float* cos,
                                const float* sin, float* rec_ml, T* rec_o, bool pdl, cudaStream_t s) {
    if (P.dc != 512 || P.dR != 64 || P.tile != kTileN) return cudaErrorInvalidValue;
    CUtensorMap tmap, tmap_rope;
    const uint64_t rows = static_cast<uint64_t>(P.kv_rows), stride = static_cast<uint64_t>(P.row_stride);
    // the tables (kv_pos_offset + max_len rows of d_R / 2 = 32 floats) are read as float4
    if (!P.rope_otf && ((reinterpret_cast<uintptr_t>(cos) | reinterpret_cast<uintptr_t>(sin)) & 15u))
        return cudaErrorInvalidValue;
    if (!make_tmap_2d_16b(&tmap, kv, rows, 576, stride, 64, 64) ||
        !make_tmap_2d_16b(&tmap_rope, kv, rows, 576, stride, 64, 8, CU_TENSOR_MAP_SWIZZLE_NONE))
        return cudaErrorInvalidValue;
    const bool paged = P.page_table != nullptr, otf = P.rope_otf != 0;
    const void* kernel = paged ? (otf ? reinterpret_cast<const void*>(decode_sm100_kernel<T, true, true>)
                                      : reinterpret_cast<const void*>(decode_sm100_kernel<T, true, false>))
                               : (otf ? reinterpret_cast<const void*>(decode_sm100_kernel<T, false, true>)
                                      : reinterpret_cast<const void*>(decode_sm100_kernel<T, false, false>));
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
    if (paged && otf)
        e = cudaLaunchKernelEx(&cfg, decode_sm100_kernel<T, true, true>, tmap, tmap_rope, P, qpack, cos, sin, rec_ml, rec_o);
    else if (paged)
        e = cudaLaunchKernelEx(&cfg, decode_sm100_kernel<T, true, false>, tmap, tmap_rope, P, qpack, cos, sin, rec_ml,
                               rec_o);
    else if (otf)
        e = cudaLaunchKernelEx(&cfg, decode_sm100_kernel<T, false, true>, tmap, tmap_rope, P, qpack, cos, sin, rec_ml,
                               rec_o);
    else
        e = cudaLaunchKernelEx(&cfg, decode_sm100_kernel<T, false, false>, tmap, tmap_rope, P, qpack, cos, sin, rec_ml,
                               rec_o);
    count_launches(1);
    return e != cudaSuccess ? e : cudaGetLastError();
}

template cudaError_t launch_decode_sm100<__half>(const DecodePlan&, const __half*, const __half*, const float*,
                                                 const float*, float*, __half*, bool, cudaStream_t);
template cudaError_t launch_decode_sm100<__nv_bfloat16>(const DecodePlan&, const __nv_bfloat16*,
                                                        const __nv_bfloat16*, const float*, const float*, float*,
                                                        __nv_bfloat16*, bool, cudaStream_t);

}  // namespace mla
