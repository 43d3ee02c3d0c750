// C++ drop-in for the reference's single-token fused launcher
// (anishesg/latent-attn src/fused_mla.cuh:11-51), implemented over mla_launch_fused.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "mla_config.cuh"

// Same fields and order as the reference's FusedMLAParams (src/fused_mla.cuh:11-34).
template <typename Elem>
struct FusedMLAParamsT {
    const Elem*  kv_cache;    // (seq_len, kv_lora_rank + qk_rope_head_dim)
    int          seq_len;
    const float* q_absorbed;  // (num_heads, kv_lora_rank) fp32
    const float* q_rope;      // (num_heads, qk_rope_head_dim) fp32
    const Elem*  W_UV;        // (num_heads * v_head_dim, kv_lora_rank)
    const float* rope_cos;    // (seq_len, qk_rope_head_dim / 2) fp32
    const float* rope_sin;
    float*       output;      // (num_heads, v_head_dim) fp32
    const MLAConfig* cfg;
};
using FusedMLAParams = FusedMLAParamsT<__half>;            // the reference's fp16 form
using FusedMLAParamsBF16 = FusedMLAParamsT<__nv_bfloat16>;

namespace latent_attn_b200 {
template <typename Elem> constexpr mla_dtype_t dtype_of();
template <> constexpr mla_dtype_t dtype_of<__half>() { return MLA_DTYPE_F16; }
template <> constexpr mla_dtype_t dtype_of<__nv_bfloat16>() { return MLA_DTYPE_BF16; }
}  // namespace latent_attn_b200

// Asynchronous on `stream`; returns cudaSuccess or an error code, never syncs
// (src/fused_mla.cu:271-296 semantics).
template <typename Elem>
inline cudaError_t launch_fused_mla(const FusedMLAParamsT<Elem>& p, cudaStream_t stream = 0) {
    mla_fused_params_t c;
    c.kv_cache = p.kv_cache;
    c.seq_len = p.seq_len;
    c.q_absorbed = p.q_absorbed;
    c.q_rope = p.q_rope;
    c.W_UV = p.W_UV;
    c.rope_cos = p.rope_cos;
    c.rope_sin = p.rope_sin;
    c.output = p.output;
    c.cfg = p.cfg ? p.cfg->c_abi() : nullptr;
    return latent_attn_b200::to_cuda_error(
        mla_launch_fused(&c, latent_attn_b200::dtype_of<Elem>(), reinterpret_cast<mla_stream_t>(stream)));
}
