// Device-side append of new latent-cache rows, one per sequence (the decode loop's write side).
//
// The reference appends through LatentKVCache::append_host (src/mla_config.cuh:58-72): two
// host-to-device copies and a stream synchronisation per token, for one sequence. Here the new
// rows are already on the device (the caller's projection wrote them), every sequence of a
// batch appends in one launch, and the lengths advance on the device, so a decode step can
// append and attend without the host in between.
//
// Row layout is the cache's own: [c_t (d_c) | k_rope (d_R)], k_rope stored unrotated (the decode
// kernels rotate it with the caller's tables).
#include "mla_internal.cuh"

namespace mla {

namespace {

// One CTA per sequence b: the row of position seq_lens[b] (contiguous: kv_offsets[b] or
// b * max_len plus the position; paged: through the page table) receives the new values, then
// seq_lens[b] advances. A sequence already holding max_len rows is left as it is and reported
// through *status (bit 0); so is a row outside the cache's kv_rows rows, from a bad page id or
// offset (bit 1).
template <typename T>
__global__ void cache_append_kernel(T* __restrict__ kv, long long stride, long long kv_rows, int dc, int dR,
                                    const T* __restrict__ c_t, const T* __restrict__ k_rope,
                                    const int64_t* __restrict__ offs, const int* __restrict__ pages, int page_rows,
                                    int max_pages, int* seq_lens, int max_len, int* status, bool vec16) {
    const int b = blockIdx.x;
    const int pos = seq_lens[b];
    __syncthreads();  // every thread has read the length before thread 0 advances it
    if (pos < 0 || pos >= max_len) {
        if (threadIdx.x == 0 && status) atomicOr(status, 1);
        return;
    }
    long long row;
    if (pages) {
        const int pg = pages[static_cast<long long>(b) * max_pages + pos / page_rows];
        row = static_cast<long long>(pg) * page_rows + pos % page_rows;
        // 64-bit arithmetic: pg + 1 must not wrap for a page id near INT_MAX
        if (pg < 0 || (static_cast<long long>(pg) + 1) * page_rows > kv_rows) {
            if (threadIdx.x == 0 && status) atomicOr(status, 2);
            return;
        }
    } else {
        row = (offs ? offs[b] : static_cast<long long>(b) * max_len) + pos;
        // a row outside the cache (a bad offset) is not written
        if (row < 0 || (kv_rows > 0 && row >= kv_rows)) {
            if (threadIdx.x == 0 && status) atomicOr(status, 2);
            return;
        }
    }
    T* dst = kv + row * stride;
    const T* src_c = c_t + static_cast<long long>(b) * dc;
    const T* src_r = k_rope + static_cast<long long>(b) * dR;
    if (vec16) {
        // 16-byte units: d_c, d_R, the stride and all base addresses are multiples of 8 elements
        const int nc = dc / 8, n = (dc + dR) / 8;
        for (int i = threadIdx.x; i < n; i += blockDim.x) {
            const uint4 v = i < nc ? reinterpret_cast<const uint4*>(src_c)[i]
                                   : reinterpret_cast<const uint4*>(src_r)[i - nc];
            reinterpret_cast<uint4*>(dst)[i] = v;
        }
    } else {
        for (int i = threadIdx.x; i < dc + dR; i += blockDim.x) dst[i] = i < dc ? src_c[i] : src_r[i - dc];
    }
    if (threadIdx.x == 0) seq_lens[b] = pos + 1;
}

}  // namespace

template <typename T>
cudaError_t launch_cache_append(T* kv, long long stride, long long kv_rows, int dc, int dR, int batch, const T* c_t,
                                const T* k_rope, const int64_t* offs, const int* pages, int page_rows, int max_pages,
                                int* seq_lens, int max_len, int* status, cudaStream_t s) {
    auto a16 = [](const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; };
    const bool vec16 = dc % 8 == 0 && dR % 8 == 0 && stride % 8 == 0 && a16(kv) && a16(c_t) && a16(k_rope);
    cache_append_kernel<T><<<batch, 128, 0, s>>>(kv, stride, kv_rows, dc, dR, c_t, k_rope, offs, pages, page_rows,
                                                 max_pages, seq_lens, max_len, status, vec16);
    count_launches(1);
    return cudaGetLastError();
}

template cudaError_t launch_cache_append<__half>(__half*, long long, long long, int, int, int, const __half*,
                                                 const __half*, const int64_t*, const int*, int, int, int*, int, int*,
                                                 cudaStream_t);
template cudaError_t launch_cache_append<__nv_bfloat16>(__nv_bfloat16*, long long, long long, int, int, int,
                                                        const __nv_bfloat16*, const __nv_bfloat16*, const int64_t*,
                                                        const int*, int, int, int*, int, int*, cudaStream_t);

}  // namespace mla
