// Weight-streaming tcgen05 GEMM for the projections around the decode (the layer-level caller of
// the reference, latent_attn/__init__.py:110-145):
//     Y[M x N] (fp32) = X[M x K] . W[N x K]^T        X, W: fp16 or bf16, row-major
// with M the decode step's tokens (1 .. 256) and N, K the model's projection sizes
// (q_absorbed: N = H * d_c, K = d_model; the output projection W_O: N = d_model, K = H * dv).
// For a decode step the weights are the bytes that matter, so the product is computed transposed,
// D^T[128 weight rows x Mp tokens] per CTA, with the 128-row weight tile as the MMA's M side and
// every token on its N side: each weight byte is read from HBM once for all tokens.
//   A = W rows [n0, n0 + 128) x 64 K, K-major, 128-byte swizzle (TMA box 64 x 128)
//   B = X rows [0, Mp) x 64 K, K-major, 128-byte swizzle (TMA box 64 x Mp; rows past M read zeros)
// streamed through a ring of (16 KB + Mp * 128 B) stages. When the N tiles alone cannot fill the
// GPU the K range is split over CTAs, which add their partial tiles into the zeroed output.
// Warp 0 (one lane) loads, warp 1 (one lane) issues the MMAs, and all 4 warps read the
// accumulator out: thread t holds weight row n0 + t, so for a token m a warp stores 32
// consecutive floats of Y's row m.
// Every wait is bounded; a wait that gives up leaves the tile's output unwritten and records a
// timeout in the library's linear-status word.
#include "mla_internal.cuh"
#include "sm100_ptx.cuh"
#include "tma_host.cuh"

namespace mla {
using namespace sm100;

namespace {
constexpr int kLinRows = 128;        // weight rows per CTA (MMA M)
constexpr int kLinChunk = 64;        // K elements per stage (one 128-byte swizzle row)
constexpr int kLinThreads = 128;
constexpr int kLinSmemCap = 200 * 1024;

template <typename T> struct LinFmt;
template <> struct LinFmt<__half> { static constexpr uint32_t v = 0; };
template <> struct LinFmt<__nv_bfloat16> { static constexpr uint32_t v = 1; };

__device__ __forceinline__ int lin_code(int site) { return kStatusTimeout | (site << 8); }

__host__ __device__ inline int lin_stage_bytes(int Mp) { return kLinRows * 128 + Mp * 128; }
}  // namespace

template <typename T>
__global__ void __launch_bounds__(kLinThreads, 1)
linear_sm100_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                    float* __restrict__ Y, int M, int N, int K, int Mp, int chunks_per_split, int stages,
                    uint32_t tmem_cols, int* status) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const int stage_bytes = lin_stage_bytes(Mp);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + stages * stage_bytes);
    uint64_t* empty = full + stages;
    uint64_t* done = empty + stages;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    const uint32_t ring = smem_u32(smem);
    const int warp = threadIdx.x >> 5;
    const int n0 = blockIdx.x * kLinRows;
    const int nchunks = (K + kLinChunk - 1) / kLinChunk;
    const int c0 = blockIdx.y * chunks_per_split;
    const int c1 = min(nchunks, c0 + chunks_per_split);
    const bool split = gridDim.y > 1;
    volatile int* err = status;

    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; ++s) {
            mbar_init(smem_u32(&full[s]), 1);
            mbar_init(smem_u32(&empty[s]), 1);
        }
        mbar_init(smem_u32(done), 1);
        fence_mbar_init();
        tma_prefetch_desc(&tmap_w);
        tma_prefetch_desc(&tmap_x);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), tmem_cols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *tmem_slot;
    pdl_wait();   // X may come from the previous kernel
    bool ok = true;

    if (threadIdx.x == 0) {
        // ---- producer
        int issued = 0;
        for (int c = c0, i = 0; c < c1; ++c, ++i) {
            const int s = i % stages;
            if (i >= stages && !mbar_wait(smem_u32(&empty[s]), ((i / stages) - 1) & 1, err, lin_code(1))) break;
            const uint32_t fb = smem_u32(&full[s]);
            mbar_arrive_expect_tx(fb, static_cast<uint32_t>(stage_bytes));
            const uint32_t dst = ring + s * stage_bytes;
            tma_load_2d(dst, &tmap_w, fb, kLinChunk * c, n0);
            tma_load_2d(dst + kLinRows * 128, &tmap_x, fb, kLinChunk * c, 0);
            issued = i + 1;
        }
        // shared memory is not released under a TMA write: the last loads land before teardown
        for (int i = issued > stages ? issued - stages : 0; i < issued; ++i)
            mbar_wait(smem_u32(&full[i % stages]), (i / stages) & 1, err, lin_code(2), 100000000ull);
    } else if (threadIdx.x == 32) {
        // ---- MMA issuer
        const uint32_t idesc = idesc_f16(kLinRows, Mp, LinFmt<T>::v, false, false);
        for (int c = c0, i = 0; c < c1; ++c, ++i) {
            const int s = i % stages;
            if (!mbar_wait(smem_u32(&full[s]), (i / stages) & 1, err, lin_code(3))) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t a = ring + s * stage_bytes, b = a + kLinRows * 128;
            const uint64_t ad = smem_desc_sw128(a, 16, 1024), bd = smem_desc_sw128(b, 16, 1024);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
                mma_ss(tbase, ad + static_cast<uint64_t>(2 * kk), bd + static_cast<uint64_t>(2 * kk), idesc,
                       (i | kk) != 0 ? 1u : 0u);
            mma_commit(smem_u32(&empty[s]));
        }
        mma_commit(smem_u32(done));   // also arrives when nothing was issued
    }
    // ---- epilogue: thread t = TMEM lane t = weight row n0 + t
    bool got = mbar_wait(smem_u32(done), 0, err, lin_code(4));
    got = __syncthreads_and(got && ok);
    if (got && c1 > c0) {
        tc_fence_after();
        const int n = n0 + threadIdx.x;
        const uint32_t trow = tbase + (static_cast<uint32_t>(32 * warp) << 16);
        for (int m0 = 0; m0 < M; m0 += 16) {
            uint32_t v[16];
            tmem_ld16_sync(trow + m0, v);
            if (n < N) {
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int m = m0 + j;
                    if (m < M) {
                        float* dst = Y + static_cast<long long>(m) * N + n;
                        if (split) atomicAdd(dst, __uint_as_float(v[j]));
                        else *dst = __uint_as_float(v[j]);
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tbase, tmem_cols);
    }
}

namespace {
// Timeouts of the projection GEMM's waits are recorded here (diagnostics; the call's result is
// otherwise incomplete output).
__device__ int g_linear_status;
}  // namespace

bool linear_sm100_supported(int M, int N, int K) {
    return M >= 1 && M <= 256 && N >= 1 && K >= 8 && K % 8 == 0;
}

template <typename T>
cudaError_t launch_linear_sm100(const T* X, const T* W, float* Y, int M, int N, int K, int sms, cudaStream_t s) {
    if (!linear_sm100_supported(M, N, K)) return cudaErrorInvalidValue;
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
            e = cudaGetSymbolAddress(&a, g_linear_status);
            if (e != cudaSuccess) return e;
            status_addr[dev] = static_cast<int*>(a);
        }
        status = status_addr[dev];
    }
    const int Mp = (M + 15) / 16 * 16;
    CUtensorMap tw, tx;
    if (!make_tmap_2d_16b(&tw, W, static_cast<uint64_t>(N), static_cast<uint64_t>(K), static_cast<uint64_t>(K),
                          kLinRows, kLinChunk) ||
        !make_tmap_2d_16b(&tx, X, static_cast<uint64_t>(M), static_cast<uint64_t>(K), static_cast<uint64_t>(K),
                          static_cast<uint32_t>(Mp), kLinChunk))
        return cudaErrorInvalidValue;
    const int stage_bytes = lin_stage_bytes(Mp);
    int stages = kLinSmemCap / stage_bytes;
    stages = stages > 8 ? 8 : (stages < 2 ? 2 : stages);
    const size_t smem = static_cast<size_t>(stages) * stage_bytes + (2 * stages + 1) * 8 + 16 + 1024;
    const int tiles = (N + kLinRows - 1) / kLinRows;
    const int nchunks = (K + kLinChunk - 1) / kLinChunk;
    // split K while the row tiles leave SMs idle, keeping at least 4 chunks per split
    int splits = (sms + tiles - 1) / tiles;
    if (splits > nchunks / 4) splits = nchunks / 4;
    if (splits < 1) splits = 1;
    const int per = (nchunks + splits - 1) / splits;
    splits = (nchunks + per - 1) / per;
    uint32_t cols = 32;
    while (cols < static_cast<uint32_t>(Mp)) cols <<= 1;
    e = ensure_dynamic_smem(reinterpret_cast<const void*>(linear_sm100_kernel<T>), static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    if (splits > 1) {
        e = cudaMemsetAsync(Y, 0, static_cast<size_t>(M) * N * sizeof(float), s);
        if (e != cudaSuccess) return e;
    }
    linear_sm100_kernel<T><<<dim3(tiles, splits), kLinThreads, smem, s>>>(tw, tx, Y, M, N, K, Mp, per, stages, cols,
                                                                           status);
    count_launches(1);
    return cudaGetLastError();
}

template cudaError_t launch_linear_sm100<__half>(const __half*, const __half*, float*, int, int, int, int,
                                                 cudaStream_t);
template cudaError_t launch_linear_sm100<__nv_bfloat16>(const __nv_bfloat16*, const __nv_bfloat16*, float*, int,
                                                        int, int, int, cudaStream_t);

}  // namespace mla
