// Peer memory for the multi-GPU exchange: CUDA IPC allocations that the other processes of the
// node map, and the put / wait kernels that move per-head partials and outputs over NVLink with
// plain stores (no TMA). The flag protocol (per-receiver block counts, a
// system-scope release store of the step counter, a bounded acquire spin) is in peer.cuh.
#include <cstdint>
#include <cstring>

#include "mla_internal.cuh"
#include "peer.cuh"
#include "sm100_ptx.cuh"

namespace mla {
namespace {

// Block (k, q): part k of slice q (rows x row_units 16-byte units) -> dst[q]; the last of the
// gridDim.x blocks of slice q signals receiver q.
__global__ void __launch_bounds__(256) peer_put_kernel(const unsigned char* src, uint32_t rows, uint32_t row_units,
                                                       size_t src_pitch, size_t src_stride, void* const* dst,
                                                       size_t dst_pitch, size_t dst_offset, const PeerSig sig) {
    const int q = blockIdx.y;
    const unsigned char* s = src + static_cast<size_t>(q) * src_stride;
    unsigned char* d = static_cast<unsigned char*>(dst[q]) + dst_offset;
    const uint32_t total = rows * row_units;
    const uint32_t per = (total + gridDim.x - 1) / gridDim.x;
    const uint32_t u0 = blockIdx.x * per, u1 = min(total, u0 + per);
    // eight 16-byte loads in flight per thread before their stores
    for (uint32_t i0 = u0 + threadIdx.x; i0 < u1; i0 += 8 * blockDim.x) {
        uint4 v[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const uint32_t i = i0 + k * blockDim.x;
            if (i < u1) {
                const uint32_t r = i / row_units, c = i - r * row_units;
                v[k] = *reinterpret_cast<const uint4*>(s + r * src_pitch + 16u * c);
            }
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const uint32_t i = i0 + k * blockDim.x;
            if (i < u1) {
                const uint32_t r = i / row_units, c = i - r * row_units;
                *reinterpret_cast<uint4*>(d + r * dst_pitch + 16u * c) = v[k];
            }
        }
    }
    peer_block_done(sig, q, gridDim.x);
}

constexpr unsigned long long kPeerWaitNs = 2000000000ull;   // 2 s

// Launched with programmatic dependent launch: it lets the next kernel start at once (that
// kernel's own griddepcontrol.wait holds it until this one ends, so it can prefetch its weights
// meanwhile), and waits for the previous kernel before advancing the step counter, which that
// kernel may still read.
__global__ void peer_wait_kernel(const int* flags, int count, int* epoch, int advance, int* status) {
    sm100::pdl_launch_dependents();
    const int target = *epoch + 1;
    bool ok = true;
    for (int i = threadIdx.x; i < count; i += blockDim.x) {
        const unsigned long long t0 = sm100::globaltimer_ns();
        while (peer_ld_acquire(flags + i) < target) {
            if (sm100::globaltimer_ns() - t0 > kPeerWaitNs) {
                ok = false;
                break;
            }
        }
    }
    if (!ok && status) atomicExch(status, 1);
    sm100::pdl_wait();
    ok = __syncthreads_and(ok);   // also: every thread read *epoch before it advances
    if (advance && ok && threadIdx.x == 0) *epoch = target;
}

}  // namespace

cudaError_t ipc_alloc(size_t bytes, void** ptr, void* handle) {
    cudaError_t e = cudaMalloc(ptr, bytes);
    if (e != cudaSuccess) return e;
    e = cudaMemset(*ptr, 0, bytes);
    if (e != cudaSuccess) return e;
    cudaIpcMemHandle_t h;
    e = cudaIpcGetMemHandle(&h, *ptr);
    if (e != cudaSuccess) return e;
    static_assert(sizeof(cudaIpcMemHandle_t) <= 64, "IPC handle size");
    std::memset(handle, 0, 64);
    std::memcpy(handle, &h, sizeof(h));
    return cudaSuccess;
}

cudaError_t ipc_open(const void* handle, void** ptr) {
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
}

cudaError_t launch_peer_put(const void* src, size_t rows, size_t row_bytes, size_t src_pitch, size_t src_stride,
                            void* const* dst, size_t dst_pitch, size_t dst_offset, int world, int blocks,
                            const PeerSig& sig, cudaStream_t s) {
    peer_put_kernel<<<dim3(blocks, world), 256, 0, s>>>(
        static_cast<const unsigned char*>(src), static_cast<uint32_t>(rows), static_cast<uint32_t>(row_bytes / 16),
        src_pitch, src_stride, dst, dst_pitch, dst_offset, sig);
    count_launches(1);
    return cudaGetLastError();
}

cudaError_t launch_peer_wait(const int* flags, int count, int* epoch, int advance, int* status, cudaStream_t s) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(32);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, peer_wait_kernel, flags, count, epoch, advance, status);
    count_launches(1);
    return e != cudaSuccess ? e : cudaGetLastError();
}

}  // namespace mla
