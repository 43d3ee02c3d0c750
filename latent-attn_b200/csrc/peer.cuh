// Device side of the peer-memory exchange: the flag protocol shared by the put kernel and by the
// kernels that store their results straight into other GPUs' memory.
//
// A sender's kernel stores its rows into receiver q's buffer with plain stores (NVLink when q is
// another GPU), and once every block bound for q has stored its part, the last of them sets
// receiver q's flag word `flag_index` to *epoch + 1 with a system-scope release store. Blocks
// count themselves per receiver in `counters` (this GPU's memory, zero between steps): after a
// block barrier, one thread per receiver fences at GPU scope and adds 1; the block that completes
// the count resets it, fences at system scope and releases the flag (see peer_count). The receiver's wait kernel spins (bounded)
// on ld.acquire.sys until every sender's word reaches *epoch + 1; its last wait of a step
// advances *epoch, so a replayed CUDA graph carries a new value each time.
#pragma once

#include <cstdint>

#include "mla_internal.cuh"

namespace mla {

__device__ __forceinline__ int peer_ld_acquire(const int* p) {
    int v;
    asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void peer_st_release(int* p, int v) {
    asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ void peer_fence_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
__device__ __forceinline__ void peer_fence_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

// One thread's count for receiver q, after a block barrier that orders the block's stores before
// it. The GPU-scope fence makes the count a release of those stores to the other blocks of this
// GPU (the barrier makes it cumulative over the whole block); the block that completes the count
// acquires every other block's release through the counter, and its system-scope fence and
// release store carry all of them (causality order is transitive across the two scopes) to the
// receiver's acquire. One system-scope fence per receiver per kernel: a system fence in every
// block stalled the export kernel on membar for several microseconds.
__device__ __forceinline__ void peer_count(const PeerSig& s, int q, unsigned int expected) {
    peer_fence_gpu();
    const unsigned int prev = atomicAdd(s.counters + q, 1u);
    if (prev + 1u == expected) {
        s.counters[q] = 0u;   // the next step's kernel starts after this one ends
        peer_fence_sys();
        peer_st_release(s.flags[q] + s.flag_index, *s.epoch + 1);
    }
}

// Called by every thread of a block once its stores bound for receiver q are issued; `expected`
// blocks of the kernel send to q.
__device__ __forceinline__ void peer_block_done(const PeerSig& s, int q, unsigned int expected) {
    __syncthreads();
    if (threadIdx.x == 0) peer_count(s, q, expected);
}

// As peer_block_done for a block that stored into every receiver q < world (world <= blockDim.x).
__device__ __forceinline__ void peer_block_done_all(const PeerSig& s, int world, unsigned int expected) {
    __syncthreads();
    if (static_cast<int>(threadIdx.x) < world) peer_count(s, threadIdx.x, expected);
}

}  // namespace mla
