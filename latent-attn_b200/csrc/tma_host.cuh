// Host-side construction of TMA tensor maps. The driver entry point
// cuTensorMapEncodeTiled is fetched through the runtime (cudaGetDriverEntryPoint),
// so the library does not link libcuda directly.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdint>
#include <mutex>

namespace mla {

inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// 2-D row-major tensor of 16-bit elements: `rows` x `cols`, row pitch `row_stride_elems`.
// Box = box_rows x box_cols (box_cols * 2 bytes must be <= 128 for 128-byte swizzle).
// Out-of-range rows/columns of a box are zero-filled by the hardware.
// Decode steps re-describe the same cache and weights call after call, so the last
// encodings are kept (keyed by every argument) and copied instead of re-encoded.
inline bool make_tmap_2d_16b(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols,
                             uint64_t row_stride_elems, uint32_t box_rows, uint32_t box_cols,
                             CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
    struct Entry {
        const void* base;
        uint64_t rows, cols, stride;
        uint32_t box_rows, box_cols;
        int swizzle;
        CUtensorMap map;
    };
    constexpr int kCache = 16;
    static std::mutex mu;
    static Entry cache[kCache];
    static int used = 0, next = 0;
    auto same = [&](const Entry& e) {
        return e.base == base && e.rows == rows && e.cols == cols && e.stride == row_stride_elems &&
               e.box_rows == box_rows && e.box_cols == box_cols && e.swizzle == static_cast<int>(swizzle);
    };
    {
        std::lock_guard<std::mutex> lk(mu);
        for (int i = 0; i < used; ++i)
            if (same(cache[i])) {
                *map = cache[i].map;
                return true;
            }
    }
    auto enc = tensor_map_encoder();
    if (!enc) return false;
    if (reinterpret_cast<uintptr_t>(base) % 16 != 0 || (row_stride_elems * 2) % 16 != 0) return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {row_stride_elems * 2};
    cuuint32_t box[2] = {box_cols, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return false;
    std::lock_guard<std::mutex> lk(mu);
    Entry& e = cache[next];
    e.base = base;
    e.rows = rows;
    e.cols = cols;
    e.stride = row_stride_elems;
    e.box_rows = box_rows;
    e.box_cols = box_cols;
    e.swizzle = static_cast<int>(swizzle);
    e.map = *map;
    next = (next + 1) % kCache;
    if (used < kCache) ++used;
    return true;
}

// 2-D row-major fp32 tensor (rows x cols, row pitch in elements).
inline bool make_tmap_2d_f32(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols,
                             uint64_t row_stride_elems, uint32_t box_rows, uint32_t box_cols,
                             CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_NONE) {
    auto enc = tensor_map_encoder();
    if (!enc) return false;
    if (reinterpret_cast<uintptr_t>(base) % 16 != 0 || (row_stride_elems * 4) % 16 != 0) return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {row_stride_elems * 4};
    cuuint32_t box[2] = {box_cols, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

}  // namespace mla
