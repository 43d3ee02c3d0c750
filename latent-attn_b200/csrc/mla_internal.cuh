// Internal definitions shared by the decode, pack and combine kernels.
//
// Work decomposition (all decode kernels):
//   * A "group" is up to 128 query rows that attend to one KV sequence. With one
//     query token per sequence (single / variable-length batch) a group is the
//     heads [128k, 128k+128) of sequence b; with a shared cache (the reference's
//     batched op, src/fused_mla_batched.cuh:5-11) the B*H rows (token, head) are
//     flattened and cut into groups of 128 that all read sequence 0.
//   * Each group's positions are cut into tiles of TILE positions. The tiles of
//     all groups are concatenated (tile_prefix) and split evenly over W workers
//     ("stream-K"): worker w owns tiles [floor(T*w/W), floor(T*(w+1)/W)).
//   * A worker writes one partial record per group it touches. Record index
//     rec(g, w) = g + w is unique because, walking tiles in order, every step to
//     the next (group, worker) piece advances g or w. The combine kernel finds
//     group g's records from the workers holding its first and last tile.
//   * A record holds, per row: m (running max, log2 units) and l (sum of 2^(s-m)) in
//     fp32 (rec_ml), and the row's sum o of 2^(s-m) * c_t (d_c elements) rounded to the
//     cache's 16-bit type (rec_o): o itself in bf16 (fp32's exponent range), o / l in fp16
//     (a convex combination of fp16 cache rows stays inside fp16's range), see RecNorm.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <mutex>
#include <vector>

namespace mla {

constexpr int kGroupRows = 128;  // query rows per group (the tcgen05 M tile)
constexpr int kMaxRopeHalf = 64;  // on-the-fly RoPE: d_R <= 128

struct DecodePlan {
    // dims
    int dc, dR, H, dn, dv;
    int row_stride;          // cache row stride in elements
    long long kv_rows;       // rows addressable from the cache pointer (bounds the TMA tensor map)
    // batch geometry
    int B;
    int shared;              // 1: all groups read sequence 0 (rows are flattened (token, head))
    int head_blocks;         // ceil(H / 128) when !shared
    int G;                   // groups
    int max_len;             // upper bound of sequence lengths
    int uniform_len;         // > 0: every sequence has this length; no prefix array
    const int* seq_lens;     // device (B,) when !uniform
    const int64_t* kv_offsets;  // device (B,) or null
    int kv_pos_offset;       // rope table row of cache row 0
    // work split
    int tile;                // positions per tile
    int W;                   // workers
    const int* tile_prefix;  // device (G + 1,) when !uniform (written by the pack kernel)
    int* status;             // device error word (0 = ok)
    // paged layout (page_table != nullptr): position p of sequence b is row
    // page_table[b * max_pages + p / page_rows] * page_rows + p % page_rows; page_rows % 64 == 0
    const int* page_table;
    int page_rows, max_pages;
    // RoPE computed in the kernels instead of read from tables (the caller passed none):
    // rope_freq[i] = theta^(-2i/d_R) rounded to fp32, i < d_R / 2 <= kMaxRopeHalf
    int rope_otf;
    float rope_freq[kMaxRopeHalf];
};

__host__ __device__ inline int ceil_div(int a, int b) { return (a + b - 1) / b; }

// Sequence index of group g.
__device__ inline int group_seq(const DecodePlan& P, int g) { return P.shared ? 0 : g / P.head_blocks; }

__device__ inline int group_len(const DecodePlan& P, int g) {
    if (P.uniform_len > 0) return P.uniform_len;
    return P.seq_lens[group_seq(P, g)];
}

// Cache row of position pos of group g, for the first position of a tile (pos a multiple of the
// tile size; a tile never crosses a page since page_rows is a multiple of 64). Contiguous layout:
// row0 + pos. Paged layout: the page id from the sequence's page-table row; an id whose page
// lies outside the cache's kv_rows rows gives -1 (the caller reads nothing and reports it).
__device__ inline int64_t tile_kv_row(const DecodePlan& P, int g, int64_t row0, int pos) {
    if (!P.page_table) return row0 + pos;
    const int b = P.shared ? 0 : g / P.head_blocks;
    const int pg = P.page_table[static_cast<int64_t>(b) * P.max_pages + pos / P.page_rows];
    const int64_t r = static_cast<int64_t>(pg) * P.page_rows;
    if (pg < 0 || r + P.page_rows > P.kv_rows) return -1;
    return r + pos % P.page_rows;
}

__device__ inline int64_t group_kv_row0(const DecodePlan& P, int g) {
    int b = group_seq(P, g);
    if (P.kv_offsets) return P.kv_offsets[b];
    return P.shared ? 0 : static_cast<int64_t>(b) * P.max_len;
}

// Number of valid rows in group g (rows beyond H, or beyond B*H when shared, are padding).
__device__ inline int group_rows(const DecodePlan& P, int g) {
    if (P.shared) {
        int total = P.B * P.H;
        int r = total - g * kGroupRows;
        return r < kGroupRows ? r : kGroupRows;
    }
    int r = P.H - (g % P.head_blocks) * kGroupRows;
    return r < kGroupRows ? r : kGroupRows;
}

// Output row (b * H + h) of row r of group g, or -1 for a padding row.
__device__ inline int group_out_row(const DecodePlan& P, int g, int r) {
    if (P.shared) {
        int f = g * kGroupRows + r;
        return f < P.B * P.H ? f : -1;
    }
    int b = g / P.head_blocks;
    int h = (g % P.head_blocks) * kGroupRows + r;
    return h < P.H ? b * P.H + h : -1;
}

__device__ inline int tile_prefix(const DecodePlan& P, int g) {
    if (P.uniform_len > 0) return g * ceil_div(P.uniform_len, P.tile);
    return P.tile_prefix[g];
}

__device__ inline int total_tiles(const DecodePlan& P) { return tile_prefix(P, P.G); }

// (32-bit division while the products stay below 2^31: T < 2^23 tiles and W <= 256 workers)
__device__ inline int worker_begin(int T, int W, int w) {
    if (T < (1 << 23) && W <= 256) return static_cast<int>(static_cast<unsigned>(T * w) / static_cast<unsigned>(W));
    return static_cast<int>((static_cast<long long>(T) * w) / W);
}

// Worker owning global tile t.
__device__ inline int worker_of_tile(int T, int W, int t) {
    if (T < (1 << 23) && W <= 256)
        return static_cast<int>(static_cast<unsigned>((t + 1) * W - 1) / static_cast<unsigned>(T));
    return static_cast<int>(((static_cast<long long>(t) + 1) * W - 1) / T);
}

// First group whose tile range contains global tile t (binary search on the prefix).
__device__ inline int group_of_tile(const DecodePlan& P, int t) {
    if (P.uniform_len > 0) return t / ceil_div(P.uniform_len, P.tile);
    int lo = 0, hi = P.G - 1;
    while (lo < hi) {  // largest g with prefix[g] <= t and prefix[g+1] > t
        int mid = (lo + hi + 1) >> 1;
        if (P.tile_prefix[mid] <= t) lo = mid; else hi = mid - 1;
    }
    // skip empty groups (prefix[g] == prefix[g+1])
    while (lo < P.G - 1 && P.tile_prefix[lo + 1] <= t) ++lo;
    return lo;
}

// The first kernel of a decode call clears the status words. The decode kernel writes them
// only after its programmatic-dependency wait on that kernel (a bad page id), or after one of
// its own waits has failed, at least a millisecond after it starts.
__device__ inline void clear_status(const DecodePlan& P) {
    if (P.status && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && threadIdx.x < 4)
        P.status[threadIdx.x] = 0;
}

// Tiles per group, prefix-summed into prefix[0 .. G] (variable-length batches).
// Run by one whole block; G is small (batch * head_blocks).
__device__ inline void write_tile_prefix(const DecodePlan& P, int* prefix) {
    __shared__ int carry;
    if (threadIdx.x == 0) carry = 0;
    __syncthreads();
    for (int base = 0; base < P.G; base += blockDim.x) {
        int g = base + threadIdx.x;
        int v = 0;
        if (g < P.G) {
            int L = P.seq_lens[group_seq(P, g)];
            L = L < 0 ? 0 : (L > P.max_len ? P.max_len : L);
            v = ceil_div(L, P.tile);
        }
        // inclusive scan across the block (simple Hillis-Steele in shared memory)
        __shared__ int buf[1024];
        buf[threadIdx.x] = v;
        __syncthreads();
        for (int off = 1; off < blockDim.x; off <<= 1) {
            int add = threadIdx.x >= off ? buf[threadIdx.x - off] : 0;
            __syncthreads();
            buf[threadIdx.x] += add;
            __syncthreads();
        }
        if (g < P.G) prefix[g + 1] = carry + buf[threadIdx.x];
        __syncthreads();
        if (threadIdx.x == blockDim.x - 1) carry += buf[threadIdx.x];
        __syncthreads();
    }
    if (threadIdx.x == 0) prefix[0] = 0;
}

__device__ inline int num_records(const DecodePlan& P) { return P.G + P.W - 1; }

// cos and sin of the on-the-fly RoPE angle pos * freq, taken as the exact product (pos below
// 2^29 times an fp32 frequency fits the 53-bit double mantissa). The angle is reduced to
// r = angle - k 2pi, |r| <= pi, in double precision (2pi's double rounding contributes below
// 1e-9 rad for k < 2^22), rounded to fp32 (1.2e-7 rad), and the hardware approximations on
// [-pi, pi] add below 4e-7: cos and sin are within 6e-7 of their exact values. The rotated key
// is then rounded to 16 bits (relative 4e-3 for bf16).
__device__ __forceinline__ void rope_sincos_exact(long long pos, float freq, float* s, float* c) {
    const double a = static_cast<double>(pos) * static_cast<double>(freq);
    const double k = rint(a * 0.15915494309189535);  // 1 / (2 pi)
    const float r = static_cast<float>(fma(-k, 6.283185307179586, a));
    __sincosf(r, s, c);
}

// cos and sin of RoPE frequency i at absolute position pos: from the caller's tables
// ((pos, d_R / 2) fp32) or, with P.rope_otf, computed.
__device__ __forceinline__ void rope_cs(const DecodePlan& P, const float* cos_tab, const float* sin_tab,
                                        long long pos, int i, float* c, float* s) {
    if (P.rope_otf) {
        rope_sincos_exact(pos, P.rope_freq[i], s, c);
    } else {
        const long long off = pos * (P.dR / 2) + i;
        *c = cos_tab[off];
        *s = sin_tab[off];
    }
}

template <typename T> struct ElemTraits;
template <> struct ElemTraits<__half> {
    static __device__ __forceinline__ float to_f(__half x) { return __half2float(x); }
    static __device__ __forceinline__ __half from_f(float x) { return __float2half_rn(x); }
    static __device__ __forceinline__ float2 to_f2(__half2 x) { return __half22float2(x); }
    using T2 = __half2;
};
template <> struct ElemTraits<__nv_bfloat16> {
    static __device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
    static __device__ __forceinline__ __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
    static __device__ __forceinline__ float2 to_f2(__nv_bfloat162 x) { return __bfloat1622float2(x); }
    using T2 = __nv_bfloat162;
};

// Partial-record o in the cache type T: the normalised o / l for fp16 (whose range an unnormalised
// sum of up to 2^31 positions could leave), the plain sum o for bf16. The merge weighs a normalised
// record by its row sum l.
template <typename T> struct RecNorm { static constexpr bool value = false; };
template <> struct RecNorm<__half> { static constexpr bool value = true; };

// Device error codes written to DecodePlan::status.
enum : int { kStatusOk = 0, kStatusTimeout = 1, kStatusBadPlan = 2, kStatusBadPage = 3 };

// Process-wide count of kernels launched by this library (mla_kernel_launch_count).
void count_launches(int n);

// How a kernel that stores into other ranks' buffers signals them (the protocol is in peer.cuh).
struct PeerSig {
    int* const* flags;       // world pointers: receiver q's flag words
    int flag_index;          // the word this sender sets in every receiver
    const int* epoch;        // this rank's step counter
    unsigned int* counters;  // world words of this GPU: blocks of the kernel done per receiver
};

// Where the partial export writes the merged partial of (token b, head h):
// - slices == 0: ml + (b H + h) * 2 holds (m, l) and o + (b H + h) * dc the latent sum;
// - slices > 0: one packed row [m, l, 0, 0, o] of dc + 4 floats, rows grouped by head slice
//   (H / slices heads a slice): at o + ((q B + b) hs + h % hs) (dc + 4) for q = h / hs, or, with
//   peer != nullptr, in slice q's receiver: peer[q] + peer_offset bytes + (b hs + h % hs) rows.
// - gather > 0 (GEMV export only): every rank q < gather receives every row, at peer[q] +
//   peer_offset + half * parity_bytes bytes + (b H + h) rows, half = (step's flag value) & 1.
// m is in natural-log units (-inf with l = 0 for an empty partial).
struct PartOut {
    float* ml;
    float* o;
    int slices;
    void* const* peer;
    size_t peer_offset;
    int gather;
    size_t parity_bytes;
    __host__ __device__ bool to_peers() const { return peer != nullptr; }   // slices > 0 with peer
    __device__ float* row(int b, int h, int B, int H, int dc) const {
        if (!slices) return nullptr;
        const int hs = H / slices, q = h / hs;
        const long long r = static_cast<long long>(b) * hs + h % hs;
        if (peer) return reinterpret_cast<float*>(static_cast<unsigned char*>(peer[q]) + peer_offset) + r * (dc + 4);
        return o + (static_cast<long long>(q) * B * hs + r) * (dc + 4);
    }
    __device__ float* ml_at(int b, int h, int B, int H, int dc) const {
        return slices ? row(b, h, B, H, dc) : ml + (static_cast<long long>(b) * H + h) * 2;
    }
    __device__ float* o_at(int b, int h, int B, int H, int dc) const {
        return slices ? row(b, h, B, H, dc) + 4 : o + (static_cast<long long>(b) * H + h) * dc;
    }
};

// The projection's output stored into every rank's buffer as well (world == 0: `out` only):
// token b's (H, dv) rows at dst[q] + offset + b * pitch bytes for every q < world.
struct PeerRows {
    void* const* dst;
    size_t offset;
    size_t pitch;
    int world;
    PeerSig sig;
};

// The one-kernel KV-range exchange (B <= 4): every rank's receive area holds two halves (selected
// by the parity of the step's flag value *epoch + 1), each of world x B x H rows of dc + 4 packed
// values [m, l, 0, 0, o], stored as 16-byte units {v0, flag, v1, flag} so that a reader sees a value
// together with the step it belongs to (8-byte halves are written atomically) and needs no separate
// flag or fence. Sender p's row of token b, head h sits at unit ((p B + b) H + h) (dc + 4) / 2.
struct LLRing {
    void* const* recv;   // world pointers: each rank's receive area (two halves of half_bytes)
    size_t half_bytes;
    int world, rank;
    int* epoch;          // this rank's step counter, advanced by the kernel's last block
    unsigned int* done;  // zeroed block counter of this GPU
    int* status;         // set to 1 when a wait for a peer's row gives up
};

// ---- kernel launchers (defined in the .cu files; return cudaGetLastError()) ----
// pack.cu
template <typename T>
cudaError_t launch_pack_q(const DecodePlan& P, const float* q_absorbed, const float* q_nope,
                          const T* W_UK, const float* q_rope, float q_scale, T* qpack,
                          int* tile_prefix_out, cudaStream_t s);
template <typename T>
cudaError_t launch_pack_zero_pad(const DecodePlan& P, T* qpack, cudaStream_t s);
// gemm_sm100.cu: tcgen05 absorption (q_nope -> qpack) and merge + W_UV projection
bool absorb_sm100_supported(const DecodePlan& P);
bool project_sm100_supported(const DecodePlan& P);
template <typename T>
cudaError_t launch_absorb_sm100(const DecodePlan& P, const float* q_nope, const T* W_UK, const float* q_rope,
                                float q_scale, T* qpack, int* tile_prefix_out, cudaStream_t s);
template <typename T>
cudaError_t launch_project_sm100(const DecodePlan& P, const float* rec_ml, const T* rec_o, const T* W_UV,
                                 float* out, bool pdl, cudaStream_t s);
// merge of gathered partial sets of [parts][B][H] rows -- (m natural-log max, l sum; l = 0 = empty)
// at part_ml + row * ml_stride and o at part_o + row * o_stride -- followed by the W_UV projection
bool project_parts_sm100_supported(int H, int dc, int dv, int parts);
// With rows.world > 0 the merged, projected rows also go to every rank (PeerRows); with
// B <= gemv_max_tokens() the GEMV kernel stores them itself, otherwise `out` is staged and a put
// kernel follows.
// With parity_epoch the sets are read at part_ml / part_o + (*parity_epoch & 1) * parity_elems
// (a double-buffered receive area; B <= 4, the GEMV kernel).
template <typename T>
cudaError_t launch_project_parts_sm100(int B, int H, int dc, int dv, int parts, const float* part_ml,
                                       const float* part_o, int ml_stride, int o_stride, const T* W_UV, float* out,
                                       const PeerRows& rows, cudaStream_t s, const int* parity_epoch = nullptr,
                                       size_t parity_elems = 0);
// Partial export of a decode's records (one merged partial per (b, h), see PartOut) by the
// GEMV merge, for B <= gemv_max_tokens(); with part.peer, slice q's receiver is signalled.
bool export_gemv_supported(const DecodePlan& P, bool gather = false);
// The one-kernel KV-range exchange after the decode kernel (B <= kGemvMaxTok): merge this rank's
// records per head, store the packed partials into every rank's LLRing area, wait for every rank's
// partials of the same head, merge them and project with W_UV into `out` (B, H, dv).
template <typename T>
cudaError_t launch_exchange_merge(const DecodePlan& P, const float* rec_ml, const T* rec_o, const T* W_UV,
                                  float* out, const LLRing& ring, cudaStream_t s);
template <typename T>
cudaError_t launch_export_gemv(const DecodePlan& P, const float* rec_ml, const T* rec_o, const PartOut& part,
                               const PeerSig& sig, bool pdl, cudaStream_t s);
int gemv_max_tokens();
// linear_sm100.cu: Y[M x N] fp32 = X[M x K] . W[N x K]^T (the layer's projections)
bool linear_sm100_supported(int M, int N, int K);
template <typename T>
cudaError_t launch_linear_sm100(const T* X, const T* W, float* Y, int M, int N, int K, int sms, cudaStream_t s);
// decode_simt.cu
template <typename T>
cudaError_t launch_decode_simt(const DecodePlan& P, const T* kv, const T* qpack, const float* cos,
                               const float* sin, float* rec_ml, T* rec_o, cudaStream_t s);
// decode_sm100.cu
// pdl: launch with a programmatic dependency on the previous kernel (its prologue and
// cache loads overlap that kernel's tail)
template <typename T>
cudaError_t launch_decode_sm100(const DecodePlan& P, const T* kv, const T* qpack, const float* cos,
                                const float* sin, float* rec_ml, T* rec_o, bool pdl, cudaStream_t s);
bool decode_sm100_available();
// cache.cu
template <typename T>
cudaError_t launch_cache_append(T* kv, long long stride, long long kv_rows, int dc, int dR, int batch, const T* c_t,
                                const T* k_rope, const int64_t* offs, const int* pages, int page_rows, int max_pages,
                                int* seq_lens, int max_len, int* status, cudaStream_t s);
// combine.cu
// out == nullptr: export one partial per (b, h) instead (PartOut); with part.peer, slice q's
// receiver is signalled once its rows have landed
template <typename T>
cudaError_t launch_combine(const DecodePlan& P, const float* rec_ml, const T* rec_o,
                           const T* W_UV, float* out, const PartOut& part, const PeerSig& sig,
                           cudaStream_t s);
template <typename T>
cudaError_t launch_combine_parts(int B, int H, int dc, int dv, int parts, const float* part_ml,
                                 const float* part_o, int ml_stride, int o_stride, const T* W_UV, float* out,
                                 cudaStream_t s);

// peer.cu: IPC allocations and the put / wait kernels of the multi-GPU exchange
cudaError_t ipc_alloc(size_t bytes, void** ptr, void* handle);
cudaError_t ipc_open(const void* handle, void** ptr);
cudaError_t launch_peer_put(const void* src, size_t rows, size_t row_bytes, size_t src_pitch, size_t src_stride,
                            void* const* dst, size_t dst_pitch, size_t dst_offset, int world, int blocks,
                            const PeerSig& sig, cudaStream_t s);
cudaError_t launch_peer_wait(const int* flags, int count, int* epoch, int advance, int* status, cudaStream_t s);

// Raises a kernel's dynamic shared-memory limit once per device: the attribute persists,
// and setting it on every launch would cost host time in every decode call.
inline cudaError_t ensure_dynamic_smem(const void* kernel, int bytes) {
    struct Entry {
        const void* kernel;
        int dev, bytes;
    };
    static std::mutex mu;
    static std::vector<Entry> done;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lk(mu);
    for (const Entry& x : done)
        if (x.kernel == kernel && x.dev == dev && x.bytes >= bytes) return cudaSuccess;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return e;
    for (Entry& x : done)
        if (x.kernel == kernel && x.dev == dev) {
            x.bytes = bytes;
            return e;
        }
    done.push_back({kernel, dev, bytes});
    return e;
}

}  // namespace mla
