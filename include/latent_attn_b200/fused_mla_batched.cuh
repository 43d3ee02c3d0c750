// C++ drop-in for the reference's batched launcher (B query tokens over one shared
// cache; anishesg/latent-attn src/fused_mla_batched.cuh:7-35), over mla_launch_batched_fused.
#pragma once
#include "fused_mla.cuh"

// Same fields and order as BatchedFusedMLAParams (src/fused_mla_batched.cuh:7-30).
template <typename Elem>
struct BatchedFusedMLAParamsT {
    const Elem*  kv_cache;    // (seq_len, kv_lora_rank + qk_rope_head_dim), shared by all tokens
    int          seq_len;
    int          batch_size;
    const float* q_absorbed;  // (batch_size, num_heads, kv_lora_rank) fp32
    const float* q_rope;      // (batch_size, num_heads, qk_rope_head_dim) fp32
    const Elem*  W_UV;        // (num_heads * v_head_dim, kv_lora_rank)
    const float* rope_cos;    // (seq_len, qk_rope_head_dim / 2) fp32
    const float* rope_sin;
    float*       output;      // (batch_size, num_heads, v_head_dim) fp32
    const MLAConfig* cfg;
};
using BatchedFusedMLAParams = BatchedFusedMLAParamsT<__half>;
using BatchedFusedMLAParamsBF16 = BatchedFusedMLAParamsT<__nv_bfloat16>;

template <typename Elem>
inline cudaError_t launch_batched_fused_mla(const BatchedFusedMLAParamsT<Elem>& p,
                                            cudaStream_t stream = 0) {
    mla_batched_fused_params_t c;
    c.kv_cache = p.kv_cache;
    c.seq_len = p.seq_len;
    c.batch_size = p.batch_size;
    c.q_absorbed = p.q_absorbed;
    c.q_rope = p.q_rope;
    c.W_UV = p.W_UV;
    c.rope_cos = p.rope_cos;
    c.rope_sin = p.rope_sin;
    c.output = p.output;
    c.cfg = p.cfg ? p.cfg->c_abi() : nullptr;
    return latent_attn_b200::to_cuda_error(mla_launch_batched_fused(
        &c, latent_attn_b200::dtype_of<Elem>(), reinterpret_cast<mla_stream_t>(stream)));
}
