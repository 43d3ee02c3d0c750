// C++ drop-in for the reference's MLAConfig / LatentKVCache
// (anishesg/latent-attn src/mla_config.cuh:7-92), implemented over the C ABI in mla.h.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime_api.h>
#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>

#include "mla.h"

struct MLAConfig {
    int d_model;
    int kv_lora_rank;       // d_c: compressed KV latent dimension
    int qk_nope_head_dim;   // per-head non-RoPE key/query dim
    int qk_rope_head_dim;   // per-head RoPE key/query dim (d_R)
    int num_heads;
    int v_head_dim;

    // DeepSeek-V2 dims (src/mla_config.cuh:16-18)
    static MLAConfig deepseek_v2() { return {5120, 512, 128, 64, 128, 128}; }
    // DeepSeek-V3 dims as the reference returns them (src/mla_config.cuh:20-23): 128 heads
    static MLAConfig deepseek_v3() { return {7168, 512, 128, 64, 128, 128}; }

    // Bytes per packed cache row [c_t | k_rope_t] in fp16 (src/mla_config.cuh:26-28)
    int bytes_per_kv_entry() const {
        return (kv_lora_rank + qk_rope_head_dim) * static_cast<int>(sizeof(__half));
    }
    size_t kv_cache_bytes(int seq_len) const {
        return static_cast<size_t>(seq_len) * bytes_per_kv_entry();
    }
    // Throws std::invalid_argument like the reference (src/mla_config.cuh:35-40).
    void validate() const {
        if (kv_lora_rank <= 0 || qk_nope_head_dim <= 0 || qk_rope_head_dim <= 0)
            throw std::invalid_argument("MLA dims must be positive");
        if (num_heads <= 0 || v_head_dim <= 0)
            throw std::invalid_argument("num_heads and v_head_dim must be positive");
    }
    const mla_config_t* c_abi() const { return reinterpret_cast<const mla_config_t*>(this); }
};

static_assert(sizeof(MLAConfig) == sizeof(mla_config_t), "MLAConfig must mirror mla_config_t");

// Packed per-position cache: row p = [c_t (kv_lora_rank) | k_rope_t (qk_rope_head_dim)],
// stride kv_lora_rank + qk_rope_head_dim elements (src/mla_config.cuh:43-92).
struct LatentKVCache {
    __half* data;
    int max_seq_len;
    int entry_stride;
    int current_len;

    LatentKVCache(__half* device_ptr, int max_len, const MLAConfig& cfg)
        : data(device_ptr), max_seq_len(max_len),
          entry_stride(cfg.kv_lora_rank + cfg.qk_rope_head_dim), current_len(0) {}

    // Append one position from host memory; blocks until the copies finish,
    // as the reference does (src/mla_config.cuh:58-72).
    void append_host(const __half* c_t, const __half* k_rope_t, const MLAConfig& cfg,
                     cudaStream_t stream = 0) {
        if (current_len >= max_seq_len) throw std::runtime_error("KV cache full");
        __half* dst = data + static_cast<size_t>(current_len) * entry_stride;
        cudaMemcpyAsync(dst, c_t, cfg.kv_lora_rank * sizeof(__half), cudaMemcpyHostToDevice, stream);
        cudaMemcpyAsync(dst + cfg.kv_lora_rank, k_rope_t, cfg.qk_rope_head_dim * sizeof(__half),
                        cudaMemcpyHostToDevice, stream);
        cudaStreamSynchronize(stream);
        ++current_len;
    }

    __host__ __device__ const __half* row(int pos) const {
        return data + static_cast<size_t>(pos) * entry_stride;
    }
    __host__ __device__ __half* row(int pos) { return data + static_cast<size_t>(pos) * entry_stride; }
};

namespace latent_attn_b200 {
// Status -> cudaError_t for the reference-shaped launchers, which return cudaError_t.
inline cudaError_t to_cuda_error(mla_status_t s) {
    switch (s) {
        case MLA_OK: return cudaSuccess;
        case MLA_ERR_INVALID_ARGUMENT:
        case MLA_ERR_WORKSPACE: return cudaErrorInvalidValue;
        case MLA_ERR_UNSUPPORTED: return cudaErrorNotSupported;
        case MLA_ERR_NO_DEVICE_CODE: return cudaErrorNoKernelImageForDevice;
        case MLA_ERR_TIMEOUT: return cudaErrorLaunchTimeout;
        default: {
            cudaError_t e = cudaGetLastError();
            return e == cudaSuccess ? cudaErrorUnknown : e;
        }
    }
}
}  // namespace latent_attn_b200
