// TEST INFRASTRUCTURE ONLY: a C entry point around the reference's own fused
// kernels (anishesg/latent-attn src/fused_mla.cu, src/fused_mla_batched.cu),
// compiled from the reference sources in place by oracle/build_ref.py into
// oracle/_ref/libref_mla.so. Only the GPU parity tests call it, to compare the
// library against the reference's kernel on identical inputs.
#include "fused_mla.cuh"
#include "fused_mla_batched.cuh"

extern "C" int ref_fused_mla(const void* kv, int seq_len, const float* q_absorbed, const float* q_rope,
                             const void* W_UV, const float* cos, const float* sin, float* out, int d_model,
                             int dc, int dn, int dR, int H, int dv, void* stream) {
    MLAConfig cfg{d_model, dc, dn, dR, H, dv};
    FusedMLAParams p;
    p.kv_cache = static_cast<const __half*>(kv);
    p.seq_len = seq_len;
    p.q_absorbed = q_absorbed;
    p.q_rope = q_rope;
    p.W_UV = static_cast<const __half*>(W_UV);
    p.rope_cos = cos;
    p.rope_sin = sin;
    p.output = out;
    p.cfg = &cfg;
    return static_cast<int>(launch_fused_mla(p, static_cast<cudaStream_t>(stream)));
}

extern "C" int ref_batched_fused_mla(const void* kv, int seq_len, int batch, const float* q_absorbed,
                                     const float* q_rope, const void* W_UV, const float* cos, const float* sin,
                                     float* out, int d_model, int dc, int dn, int dR, int H, int dv, void* stream) {
    MLAConfig cfg{d_model, dc, dn, dR, H, dv};
    BatchedFusedMLAParams p;
    p.kv_cache = static_cast<const __half*>(kv);
    p.seq_len = seq_len;
    p.batch_size = batch;
    p.q_absorbed = q_absorbed;
    p.q_rope = q_rope;
    p.W_UV = static_cast<const __half*>(W_UV);
    p.rope_cos = cos;
    p.rope_sin = sin;
    p.output = out;
    p.cfg = &cfg;
    return static_cast<int>(launch_batched_fused_mla(p, static_cast<cudaStream_t>(stream)));
}
