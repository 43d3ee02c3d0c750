// C ABI implementation: argument validation, work planning, workspace layout and
// the launch sequence  pack(Q) -> decode(split-KV partial records) -> combine(+W_UV).
//
// Error behaviour mirrors the reference's layers: configuration errors are the
// conditions of MLAConfig::validate (src/mla_config.cuh:35-40), shape/pointer
// errors those the torch binding rejects (csrc/bindings.cpp:28-40, 146-152,
// 208-221); here they become status codes with a thread-local message instead of
// exceptions, and nothing ever exits, aborts or synchronises the host.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "latent_attn_b200/mla.h"
#include "mla_internal.cuh"
#include "peer.cuh"

struct mla_timer_st {
    cudaEvent_t begin = nullptr, end = nullptr;
    bool recorded = false;
};

namespace mla {
static std::atomic<uint64_t> g_launches{0};
void count_launches(int n) { g_launches.fetch_add(static_cast<uint64_t>(n), std::memory_order_relaxed); }
}  // namespace mla

namespace {

thread_local std::string g_last_error;

mla_status_t fail(mla_status_t s, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return s;
}

mla_status_t cuda_fail(cudaError_t e, const char* what) {
    return fail(MLA_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

struct DeviceInfo {
    int sms = 0, major = 0, minor = 0;
};

bool device_info(DeviceInfo* out) {
    static std::mutex mu;
    static std::vector<DeviceInfo> cache;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    std::lock_guard<std::mutex> lk(mu);
    if (static_cast<int>(cache.size()) <= dev) cache.resize(dev + 1);
    DeviceInfo& d = cache[dev];
    if (d.sms == 0) {
        if (cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&d.minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess) {
            d.sms = 0;
            return false;
        }
    }
    *out = d;
    return true;
}

// LATENT_ATTN_B200_PATH = "simt" | "tc" overrides the automatic kernel choice.
int env_path_override() {
    static int v = [] {
        const char* s = std::getenv("LATENT_ATTN_B200_PATH");
        if (!s) return 0;
        if (!std::strcmp(s, "tc")) return 1;
        if (!std::strcmp(s, "simt")) return 2;
        return 0;
    }();
    return v;
}

// LATENT_ATTN_B200_WORKERS = n caps the split-KV worker count (0 / unset: the planner's choice).
int env_workers() {
    static int v = [] {
        const char* s = std::getenv("LATENT_ATTN_B200_WORKERS");
        return s ? std::atoi(s) : 0;
    }();
    return v;
}

bool env_gemm_enabled() {
    static bool v = [] {
        const char* s = std::getenv("LATENT_ATTN_B200_GEMM");
        return !(s && !std::strcmp(s, "0"));
    }();
    return v;
}

constexpr size_t kAlign = 256;
size_t align_up(size_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

struct Plan {
    mla::DecodePlan dp;
    bool use_tc = false;
    bool use_gemm_absorb = false;   // tcgen05 absorption (gemm_sm100.cu) instead of the CUDA-core pack
    bool use_gemm_project = false;  // tcgen05 merge + W_UV projection instead of the CUDA-core combine
    size_t off_prefix = 0, off_qpack = 0, off_rec_ml = 0, off_rec_o = 0, off_status = 0, total = 0;
    float q_scale = 0.f;
    int nrec = 0;
};

mla_status_t validate_cfg(const mla_config_t* c) {
    if (!c) return fail(MLA_ERR_INVALID_ARGUMENT, "cfg is null");
    if (c->kv_lora_rank <= 0 || c->qk_nope_head_dim <= 0 || c->qk_rope_head_dim <= 0)
        return fail(MLA_ERR_INVALID_ARGUMENT, "MLA dims must be positive");
    if (c->num_heads <= 0 || c->v_head_dim <= 0)
        return fail(MLA_ERR_INVALID_ARGUMENT, "num_heads and v_head_dim must be positive");
    return MLA_OK;
}

// max_workers > 0 caps the split-KV worker count (the allocation-free entry point
// uses it to fit its fixed scratch array); 0 keeps the planner's own choice.
mla_status_t make_plan(const mla_config_t* cfg, const mla_decode_args_t* a, Plan* p, int max_workers = 0) {
    mla_status_t st = validate_cfg(cfg);
    if (st != MLA_OK) return st;
    if (!a) return fail(MLA_ERR_INVALID_ARGUMENT, "args is null");
    const int dc = cfg->kv_lora_rank, dR = cfg->qk_rope_head_dim, H = cfg->num_heads;
    const int dn = cfg->qk_nope_head_dim, dv = cfg->v_head_dim;
    if (a->dtype != MLA_DTYPE_F16 && a->dtype != MLA_DTYPE_BF16)
        return fail(MLA_ERR_UNSUPPORTED, "dtype must be F16 or BF16 (got %d)", static_cast<int>(a->dtype));
    if (dR % 2 != 0) return fail(MLA_ERR_UNSUPPORTED, "qk_rope_head_dim must be even (got %d)", dR);
    if (dc % 32 != 0 || dc > 1024)
        return fail(MLA_ERR_UNSUPPORTED, "kv_lora_rank must be a multiple of 32 and <= 1024 (got %d)", dc);
    if (dR > 256) return fail(MLA_ERR_UNSUPPORTED, "qk_rope_head_dim must be <= 256 (got %d)", dR);
    if (dv > 256) return fail(MLA_ERR_UNSUPPORTED, "v_head_dim must be <= 256 (got %d)", dv);
    if (a->batch <= 0) return fail(MLA_ERR_INVALID_ARGUMENT, "batch_size must be positive, got %d", a->batch);
    if (a->max_seq_len <= 0) return fail(MLA_ERR_INVALID_ARGUMENT, "max_seq_len must be positive, got %d", a->max_seq_len);
    if (a->kv_pos_offset < 0) return fail(MLA_ERR_INVALID_ARGUMENT, "kv_pos_offset must be >= 0");
    if (!a->kv_cache) return fail(MLA_ERR_INVALID_ARGUMENT, "kv_cache is null");
    if (!a->q_rope) return fail(MLA_ERR_INVALID_ARGUMENT, "q_rope is null");
    if (!a->W_UV) return fail(MLA_ERR_INVALID_ARGUMENT, "W_UV is null");
    if ((a->rope_cos == nullptr) != (a->rope_sin == nullptr))
        return fail(MLA_ERR_INVALID_ARGUMENT, "give both rope_cos and rope_sin, or neither (on-the-fly RoPE)");
    const bool rope_otf = a->rope_cos == nullptr;
    if (rope_otf && dR > 2 * mla::kMaxRopeHalf)
        return fail(MLA_ERR_UNSUPPORTED, "on-the-fly RoPE needs qk_rope_head_dim <= %d (got %d)",
                    2 * mla::kMaxRopeHalf, dR);
    if (rope_otf && a->rope_theta < 0.f) return fail(MLA_ERR_INVALID_ARGUMENT, "rope_theta must be >= 0");
    if (!a->q_absorbed && !(a->q_nope && a->W_UK))
        return fail(MLA_ERR_INVALID_ARGUMENT, "give q_absorbed, or q_nope together with W_UK");
    const int64_t stride = a->kv_row_stride ? a->kv_row_stride : (dc + dR);
    if (stride < dc + dR) return fail(MLA_ERR_INVALID_ARGUMENT, "kv_row_stride %lld < d_c + d_R", (long long)stride);
    if (stride % 8 != 0 || stride > (1 << 30))
        return fail(MLA_ERR_UNSUPPORTED, "kv_row_stride must be a multiple of 8 elements (got %lld)", (long long)stride);
    if (reinterpret_cast<uintptr_t>(a->kv_cache) % 16 != 0)
        return fail(MLA_ERR_INVALID_ARGUMENT, "kv_cache must be 16-byte aligned");
    if (reinterpret_cast<uintptr_t>(a->W_UV) % 16 != 0 || (a->W_UK && reinterpret_cast<uintptr_t>(a->W_UK) % 16 != 0))
        return fail(MLA_ERR_INVALID_ARGUMENT, "W_UV / W_UK must be 16-byte aligned");
    if (a->shared_cache && a->kv_offsets)
        return fail(MLA_ERR_INVALID_ARGUMENT, "kv_offsets must be null with shared_cache");

    mla::DecodePlan& d = p->dp;
    std::memset(&d, 0, sizeof(d));
    d.dc = dc; d.dR = dR; d.H = H; d.dn = dn; d.dv = dv;
    d.row_stride = static_cast<int>(stride);
    d.B = a->batch;
    d.shared = a->shared_cache ? 1 : 0;
    d.head_blocks = mla::ceil_div(H, mla::kGroupRows);
    if (d.shared) {
        long long rows = static_cast<long long>(a->batch) * H;
        d.G = static_cast<int>((rows + mla::kGroupRows - 1) / mla::kGroupRows);
    } else {
        d.G = a->batch * d.head_blocks;
    }
    d.max_len = a->max_seq_len;
    d.kv_offsets = a->kv_offsets;
    d.kv_pos_offset = a->kv_pos_offset;
    if (rope_otf) {
        // freq_i = theta^(-2i/d_R) (latent_attn/__init__.py:34-36 of the reference), the
        // double-precision power rounded once to fp32
        const double theta = a->rope_theta > 0.f ? static_cast<double>(a->rope_theta) : 10000.0;
        d.rope_otf = 1;
        for (int i = 0; i < dR / 2; ++i)
            d.rope_freq[i] = static_cast<float>(std::pow(theta, -2.0 * i / static_cast<double>(dR)));
    }
    if (a->kv_total_rows < 0) return fail(MLA_ERR_INVALID_ARGUMENT, "kv_total_rows must be >= 0");
    if (a->page_table) {
        if (a->shared_cache || a->kv_offsets)
            return fail(MLA_ERR_INVALID_ARGUMENT, "page_table excludes shared_cache and kv_offsets");
        if (a->page_rows <= 0 || a->page_rows % 64 != 0)
            return fail(MLA_ERR_UNSUPPORTED, "page_rows must be a positive multiple of 64, got %d", a->page_rows);
        if (static_cast<long long>(a->max_pages) * a->page_rows < a->max_seq_len)
            return fail(MLA_ERR_INVALID_ARGUMENT, "max_pages %d x page_rows %d < max_seq_len %d", a->max_pages,
                        a->page_rows, a->max_seq_len);
        if (a->kv_total_rows <= 0)
            return fail(MLA_ERR_INVALID_ARGUMENT, "kv_total_rows (rows of the page pool) is required with page_table");
        d.page_table = a->page_table;
        d.page_rows = a->page_rows;
        d.max_pages = a->max_pages;
    }
    if (a->kv_total_rows > 0) d.kv_rows = a->kv_total_rows;
    else if (a->kv_offsets) return fail(MLA_ERR_INVALID_ARGUMENT, "kv_total_rows is required with kv_offsets");
    else d.kv_rows = d.shared ? a->max_seq_len : static_cast<long long>(a->batch) * a->max_seq_len;
    const bool uniform = a->seq_lens == nullptr || d.shared;
    if (d.shared && a->seq_lens)
        return fail(MLA_ERR_INVALID_ARGUMENT, "seq_lens must be null with shared_cache (one sequence)");
    d.uniform_len = uniform ? a->max_seq_len : 0;
    d.seq_lens = a->seq_lens;

    DeviceInfo di;
    if (!device_info(&di)) return fail(MLA_ERR_CUDA, "no CUDA device");
    const bool tc_shape = dc == 512 && dR == 64;
    bool use_tc = tc_shape && di.major == 10 && mla::decode_sm100_available();
    int ov = a->kernel != MLA_KERNEL_AUTO ? a->kernel : env_path_override();
    if (ov == 2) use_tc = false;
    if (ov == 1) {
        if (!tc_shape || di.major != 10 || !mla::decode_sm100_available())
            return fail(MLA_ERR_UNSUPPORTED, "tensor-core path forced but unavailable for this shape/device");
        use_tc = true;
    }
    p->use_tc = use_tc;
    d.tile = use_tc ? 64 : 32;

    // tiles, if known on the host
    long long T = -1;
    if (uniform) {
        T = static_cast<long long>(d.G) * mla::ceil_div(a->max_seq_len, d.tile);
    } else if (a->seq_lens_host) {
        T = 0;
        for (int b = 0; b < a->batch; ++b) {
            int L = a->seq_lens_host[b];
            if (L < 0 || L > a->max_seq_len)
                return fail(MLA_ERR_INVALID_ARGUMENT, "seq_lens[%d]=%d outside [0, max_seq_len=%d]", b, L, a->max_seq_len);
            T += static_cast<long long>(d.head_blocks) * mla::ceil_div(L, d.tile);
        }
    }
    if (T > (1LL << 30)) return fail(MLA_ERR_UNSUPPORTED, "too many positions");
    int cap = use_tc ? di.sms / 2 : 64;
    if (cap > 128) cap = 128;  // the combine kernel merges at most 128 records per row
    if (max_workers > 0 && cap > max_workers) cap = max_workers;
    if (env_workers() > 0 && cap > env_workers()) cap = env_workers();
    if (cap < 1) cap = 1;
    int W = cap;
    if (T >= 0 && T < W) W = T > 0 ? static_cast<int>(T) : 1;
    d.W = W;
    p->nrec = d.G + W - 1;

    size_t off = 0;
    p->off_status = off; off = align_up(off + sizeof(int) * 4);
    p->off_prefix = off; off = align_up(off + sizeof(int) * (static_cast<size_t>(d.G) + 1));
    p->off_qpack = off;
    off = align_up(off + static_cast<size_t>(d.G) * mla::kGroupRows * (dc + dR) * 2);
    p->off_rec_ml = off;
    off = align_up(off + static_cast<size_t>(p->nrec) * mla::kGroupRows * 2 * sizeof(float));
    p->off_rec_o = off;   // o / l rows in the cache's 16-bit type
    off = align_up(off + static_cast<size_t>(p->nrec) * mla::kGroupRows * dc * 2);
    p->total = off;

    // the tcgen05 GEMMs run on sm_100 whenever their shape constraints hold
    // (LATENT_ATTN_B200_GEMM=0 keeps the CUDA-core pack / combine kernels)
    const bool gemm_ok = di.major == 10 && env_gemm_enabled();
    p->use_gemm_absorb = gemm_ok && mla::absorb_sm100_supported(d);
    p->use_gemm_project = gemm_ok && mla::project_sm100_supported(d);

    float scale = a->softmax_scale > 0.f ? a->softmax_scale : 1.0f / std::sqrt(static_cast<float>(dn + dR));
    p->q_scale = scale * 1.4426950408889634f;  // log2(e): scores in log2 units
    return MLA_OK;
}

// Timer event record. Under stream capture it must be an external record, which becomes a
// graph node that fires on every replay (a plain record would only express a dependency);
// outside capture the external flag is not accepted, so a plain record is used.
cudaError_t timer_record(cudaEvent_t ev, cudaStream_t s) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaError_t e = cudaStreamIsCapturing(s, &cs);
    if (e != cudaSuccess) return e;
    return cs == cudaStreamCaptureStatusActive ? cudaEventRecordWithFlags(ev, s, cudaEventRecordExternal)
                                               : cudaEventRecord(ev, s);
}

template <typename T>
mla_status_t run_decode(const Plan& pl, const mla_decode_args_t* a, unsigned char* ws, float* out,
                        const mla::PartOut& part, const mla::PeerSig& sig, cudaStream_t s,
                        const mla::LLRing* ring = nullptr) {
    mla::DecodePlan d = pl.dp;
    int* prefix = reinterpret_cast<int*>(ws + pl.off_prefix);
    d.tile_prefix = d.uniform_len > 0 ? nullptr : prefix;
    d.status = reinterpret_cast<int*>(ws + pl.off_status);
    T* qpack = reinterpret_cast<T*>(ws + pl.off_qpack);
    float* rec_ml = reinterpret_cast<float*>(ws + pl.off_rec_ml);
    T* rec_o = reinterpret_cast<T*>(ws + pl.off_rec_o);
    // the status words are cleared by the first kernel below (clear_status)
    cudaError_t e = cudaSuccess;
    int* prefix_out = d.uniform_len > 0 ? nullptr : prefix;
    if (!a->q_absorbed && pl.use_gemm_absorb) {
        e = mla::launch_pack_zero_pad<T>(d, qpack, s);
        if (e == cudaSuccess)
            e = mla::launch_absorb_sm100<T>(d, a->q_nope, reinterpret_cast<const T*>(a->W_UK), a->q_rope, pl.q_scale,
                                            qpack, prefix_out, s);
        if (e != cudaSuccess) return cuda_fail(e, "absorption kernel launch");
    } else {
        e = mla::launch_pack_q<T>(d, a->q_absorbed, a->q_absorbed ? nullptr : a->q_nope,
                                  reinterpret_cast<const T*>(a->W_UK), a->q_rope, pl.q_scale, qpack, prefix_out, s);
        if (e != cudaSuccess) return cuda_fail(e, "pack kernel launch");
    }
    const T* kv = reinterpret_cast<const T*>(a->kv_cache);
    if (a->timer) {
        e = timer_record(a->timer->begin, s);
        if (e != cudaSuccess) return cuda_fail(e, "cudaEventRecord(timer)");
    }
    // with a timer the decode kernel must not overlap the packing kernel, so that the
    // events bracket it exactly
    if (pl.use_tc)
        e = mla::launch_decode_sm100<T>(d, kv, qpack, a->rope_cos, a->rope_sin, rec_ml, rec_o, a->timer == nullptr, s);
    else
        e = mla::launch_decode_simt<T>(d, kv, qpack, a->rope_cos, a->rope_sin, rec_ml, rec_o, s);
    if (e == cudaErrorNoKernelImageForDevice || e == cudaErrorInvalidDeviceFunction)
        return fail(MLA_ERR_NO_DEVICE_CODE, "decode kernel: %s (library is built for sm_100a)", cudaGetErrorString(e));
    if (e != cudaSuccess) return cuda_fail(e, "decode kernel launch");
    if (a->timer) {
        e = timer_record(a->timer->end, s);
        if (e != cudaSuccess) return cuda_fail(e, "cudaEventRecord(timer)");
        a->timer->recorded = true;
    }
    if (ring) {
        if (!pl.use_gemm_project)
            return fail(MLA_ERR_UNSUPPORTED, "the KV-range exchange needs the tensor-core path (sm_100)");
        e = mla::launch_exchange_merge<T>(d, rec_ml, rec_o, reinterpret_cast<const T*>(a->W_UV), out, *ring, s);
    } else if (out && pl.use_gemm_project)
        e = mla::launch_project_sm100<T>(d, rec_ml, rec_o, reinterpret_cast<const T*>(a->W_UV), out, true, s);
    else if (!out && pl.use_gemm_project && mla::export_gemv_supported(d, part.gather > 0))
        e = mla::launch_export_gemv<T>(d, rec_ml, rec_o, part, sig, true, s);
    else if (part.gather > 0)
        return fail(MLA_ERR_UNSUPPORTED, "the gathered export needs the tensor-core path and batch <= 4");
    else
        e = mla::launch_combine<T>(d, rec_ml, rec_o, reinterpret_cast<const T*>(a->W_UV), out, part, sig, s);
    if (e != cudaSuccess) return cuda_fail(e, "combine kernel launch");
    return MLA_OK;
}

mla_status_t decode_impl(const mla_config_t* cfg, const mla_decode_args_t* a, void* workspace,
                         size_t ws_bytes, float* out, const mla::PartOut& part, cudaStream_t s,
                         int max_workers = 0, const mla::PeerSig& sig = mla::PeerSig{},
                         const mla::LLRing* ring = nullptr) {
    Plan pl;
    mla_status_t st = make_plan(cfg, a, &pl, max_workers);
    if (st != MLA_OK) return st;
    if (!workspace) return fail(MLA_ERR_WORKSPACE, "workspace is null");
    if (reinterpret_cast<uintptr_t>(workspace) % kAlign != 0)
        return fail(MLA_ERR_WORKSPACE, "workspace must be %zu-byte aligned", kAlign);
    if (ws_bytes < pl.total)
        return fail(MLA_ERR_WORKSPACE, "workspace too small: %zu < %zu bytes", ws_bytes, pl.total);
    unsigned char* ws = static_cast<unsigned char*>(workspace);
    if (a->dtype == MLA_DTYPE_BF16) return run_decode<__nv_bfloat16>(pl, a, ws, out, part, sig, s, ring);
    return run_decode<__half>(pl, a, ws, out, part, sig, s, ring);
}

// Scratch for the reference-shaped launchers, whose signatures carry no workspace.
mla_status_t decode_with_pool(const mla_config_t* cfg, const mla_decode_args_t* a, cudaStream_t s) {
    Plan pl;
    mla_status_t st = make_plan(cfg, a, &pl);
    if (st != MLA_OK) return st;
    void* ws = nullptr;
    cudaError_t e = cudaMallocAsync(&ws, pl.total, s);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMallocAsync(workspace)");
    st = decode_impl(cfg, a, ws, pl.total, a->output, mla::PartOut{}, s);
    e = cudaFreeAsync(ws, s);
    if (st == MLA_OK && e != cudaSuccess) return cuda_fail(e, "cudaFreeAsync(workspace)");
    return st;
}

// ---------------------------------------------------------------------------
// Allocation-free variant of the single-token launcher.
//
// Its split-KV scratch (status word, packed query, partial records) lives in one
// file-scope device array instead of memory from cudaMalloc / cudaMallocAsync.
// In host code the array's name is only a stand-in for the device symbol, so the
// real device address is looked up with cudaGetSymbolAddress, once per device,
// with that device current, and passed to the kernels.
// ---------------------------------------------------------------------------
static __device__ __align__(256) unsigned char g_noalloc_scratch[MLA_NOALLOC_SCRATCH_BYTES];

// Device address of g_noalloc_scratch on the current device (looked up once per device).
mla_status_t noalloc_scratch(void** out) {
    static std::mutex mu;
    static std::vector<void*> addr;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    std::lock_guard<std::mutex> lk(mu);
    if (static_cast<int>(addr.size()) <= dev) addr.resize(dev + 1, nullptr);
    if (!addr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(static scratch)");
        addr[dev] = p;
    }
    *out = addr[dev];
    return MLA_OK;
}

// Merge `num_parts` partial sets of (B, heads) rows and project with W_UV (heads * dv, d_c):
// m, l at part_ml + row * ml_stride, o at part_o + row * o_stride. With rows.world > 0 the
// output also goes to every rank (the GEMV kernel stores it itself; otherwise `output` stages it
// for a put kernel).
mla_status_t combine_impl(const mla_config_t* cfg, mla_dtype_t dtype, int batch, int num_parts, int heads,
                          const float* part_ml, const float* part_o, int ml_stride, int o_stride,
                          const void* W_UV, float* output, cudaStream_t s, const mla::PeerRows& rows = mla::PeerRows{},
                          const int* parity_epoch = nullptr, size_t parity_elems = 0) {
    mla_status_t st = validate_cfg(cfg);
    if (st != MLA_OK) return st;
    if (batch <= 0 || num_parts <= 0 || heads <= 0)
        return fail(MLA_ERR_INVALID_ARGUMENT, "batch, num_parts and heads must be positive");
    if (!part_ml || !part_o || !W_UV || !output) return fail(MLA_ERR_INVALID_ARGUMENT, "null pointer");
    if (cfg->kv_lora_rank > 1024 || cfg->v_head_dim > 256)
        return fail(MLA_ERR_UNSUPPORTED, "kv_lora_rank <= 1024 and v_head_dim <= 256 required");
    if (dtype != MLA_DTYPE_BF16 && dtype != MLA_DTYPE_F16) return fail(MLA_ERR_UNSUPPORTED, "dtype must be F16 or BF16");
    DeviceInfo di;
    if (!device_info(&di)) return fail(MLA_ERR_CUDA, "no CUDA device");
    const int dc = cfg->kv_lora_rank, dv = cfg->v_head_dim;
    // tcgen05 merge + W_UV GEMM when the shape fits, else the CUDA-core combine
    const bool gemm = di.major == 10 && (env_gemm_enabled() || parity_epoch) &&
                      mla::project_parts_sm100_supported(heads, dc, dv, num_parts);
    if (parity_epoch && (!gemm || batch > 4))
        return fail(MLA_ERR_UNSUPPORTED, "gathered partial sets need an sm_100 GPU, batch <= 4, v_head_dim 128, "
                                         "kv_lora_rank a multiple of 64 up to 512 and at most 128 parts");
    cudaError_t e;
    if (gemm && dtype == MLA_DTYPE_BF16)
        e = mla::launch_project_parts_sm100<__nv_bfloat16>(batch, heads, dc, dv, num_parts, part_ml, part_o, ml_stride,
                                                          o_stride, static_cast<const __nv_bfloat16*>(W_UV), output,
                                                          rows, s, parity_epoch, parity_elems);
    else if (gemm)
        e = mla::launch_project_parts_sm100<__half>(batch, heads, dc, dv, num_parts, part_ml, part_o, ml_stride, o_stride,
                                                   static_cast<const __half*>(W_UV), output, rows, s, parity_epoch,
                                                   parity_elems);
    else {
        if (dtype == MLA_DTYPE_BF16)
            e = mla::launch_combine_parts<__nv_bfloat16>(batch, heads, dc, dv, num_parts, part_ml, part_o, ml_stride,
                                                         o_stride, static_cast<const __nv_bfloat16*>(W_UV), output, s);
        else
            e = mla::launch_combine_parts<__half>(batch, heads, dc, dv, num_parts, part_ml, part_o, ml_stride, o_stride,
                                                  static_cast<const __half*>(W_UV), output, s);
        if (e == cudaSuccess && rows.world > 0) {
            const size_t row_bytes = static_cast<size_t>(heads) * dv * sizeof(float);
            const int blocks = static_cast<int>(std::min<size_t>(32, (batch * row_bytes + 16383) / 16384));
            e = mla::launch_peer_put(output, batch, row_bytes, row_bytes, 0, rows.dst, rows.pitch, rows.offset,
                                     rows.world, blocks, rows.sig, s);
        }
    }
    if (e != cudaSuccess) return cuda_fail(e, "combine kernel launch");
    return MLA_OK;
}

}  // namespace

namespace {
// The signal description of a kernel that stores into other ranks' buffers.
mla_status_t peer_sig(const mla_peer_signal_t* in, mla::PeerSig* out) {
    if (!in || !in->flags || !in->epoch || !in->counters)
        return fail(MLA_ERR_INVALID_ARGUMENT, "peer signal: flags, epoch and counters must be non-null");
    if (in->flag_index < 0) return fail(MLA_ERR_INVALID_ARGUMENT, "peer signal: flag_index must be >= 0");
    *out = mla::PeerSig{in->flags, in->flag_index, in->epoch, in->counters};
    return MLA_OK;
}
}  // namespace

extern "C" {

mla_status_t mla_config_validate(const mla_config_t* cfg) { return validate_cfg(cfg); }

mla_status_t mla_decode_workspace_size(const mla_config_t* cfg, const mla_decode_args_t* a, size_t* bytes) {
    if (!bytes) return fail(MLA_ERR_INVALID_ARGUMENT, "bytes is null");
    Plan pl;
    mla_status_t st = make_plan(cfg, a, &pl);
    if (st != MLA_OK) return st;
    *bytes = pl.total;
    return MLA_OK;
}

mla_status_t mla_decode(const mla_config_t* cfg, const mla_decode_args_t* a, void* workspace,
                        size_t workspace_bytes, mla_stream_t stream) {
    if (!a) return fail(MLA_ERR_INVALID_ARGUMENT, "args is null");
    if (!a->output) return fail(MLA_ERR_INVALID_ARGUMENT, "output is null");
    return decode_impl(cfg, a, workspace, workspace_bytes, a->output, mla::PartOut{},
                       reinterpret_cast<cudaStream_t>(stream));
}

mla_status_t mla_decode_partial(const mla_config_t* cfg, const mla_decode_args_t* a, float* partial_ml,
                                float* partial_o, void* workspace, size_t workspace_bytes,
                                mla_stream_t stream) {
    if (!partial_ml || !partial_o) return fail(MLA_ERR_INVALID_ARGUMENT, "partial outputs are null");
    return decode_impl(cfg, a, workspace, workspace_bytes, nullptr, mla::PartOut{partial_ml, partial_o, 0, nullptr, 0},
                       reinterpret_cast<cudaStream_t>(stream));
}

mla_status_t mla_combine_partials(const mla_config_t* cfg, mla_dtype_t dtype, int batch, int num_parts,
                                  const float* partial_ml, const float* partial_o, const void* W_UV,
                                  float* output, mla_stream_t stream) {
    mla_status_t st = validate_cfg(cfg);
    if (st != MLA_OK) return st;
    return combine_impl(cfg, dtype, batch, num_parts, cfg->num_heads, partial_ml, partial_o, 2, cfg->kv_lora_rank, W_UV,
                        output, reinterpret_cast<cudaStream_t>(stream));
}

mla_status_t mla_linear(mla_dtype_t dtype, int M, int N, int K, const void* X, const void* W, float* Y,
                        mla_stream_t stream) {
    if (!X || !W || !Y) return fail(MLA_ERR_INVALID_ARGUMENT, "null pointer");
    if (M <= 0 || N <= 0 || K <= 0) return fail(MLA_ERR_INVALID_ARGUMENT, "M, N and K must be positive");
    if (dtype != MLA_DTYPE_BF16 && dtype != MLA_DTYPE_F16) return fail(MLA_ERR_UNSUPPORTED, "dtype must be F16 or BF16");
    if (!mla::linear_sm100_supported(M, N, K))
        return fail(MLA_ERR_UNSUPPORTED, "mla_linear needs 1 <= M <= 256 and K a multiple of 8 (M=%d, K=%d)", M, K);
    if ((reinterpret_cast<uintptr_t>(X) | reinterpret_cast<uintptr_t>(W)) % 16 != 0)
        return fail(MLA_ERR_INVALID_ARGUMENT, "X and W must be 16-byte aligned");
    DeviceInfo di;
    if (!device_info(&di)) return fail(MLA_ERR_CUDA, "no CUDA device");
    if (di.major != 10) return fail(MLA_ERR_NO_DEVICE_CODE, "mla_linear needs an sm_100 GPU");
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    cudaError_t e = dtype == MLA_DTYPE_BF16
                        ? mla::launch_linear_sm100<__nv_bfloat16>(static_cast<const __nv_bfloat16*>(X),
                                                                  static_cast<const __nv_bfloat16*>(W), Y, M, N, K,
                                                                  di.sms, s)
                        : mla::launch_linear_sm100<__half>(static_cast<const __half*>(X), static_cast<const __half*>(W),
                                                           Y, M, N, K, di.sms, s);
    if (e == cudaErrorNoKernelImageForDevice || e == cudaErrorInvalidDeviceFunction)
        return fail(MLA_ERR_NO_DEVICE_CODE, "linear kernel: %s (library is built for sm_100a)", cudaGetErrorString(e));
    if (e != cudaSuccess) return cuda_fail(e, "linear kernel launch");
    return MLA_OK;
}

mla_status_t mla_decode_partial_packed(const mla_config_t* cfg, const mla_decode_args_t* a, int num_slices,
                                       float* packed, void* workspace, size_t workspace_bytes, mla_stream_t stream) {
    mla_status_t st = validate_cfg(cfg);
    if (st != MLA_OK) return st;
    if (!packed) return fail(MLA_ERR_INVALID_ARGUMENT, "packed output is null");
    if (num_slices <= 0 || cfg->num_heads % num_slices != 0)
        return fail(MLA_ERR_INVALID_ARGUMENT, "num_slices (%d) must divide num_heads (%d)", num_slices, cfg->num_heads);
    if (reinterpret_cast<uintptr_t>(packed) % 16 != 0) return fail(MLA_ERR_INVALID_ARGUMENT, "packed must be 16-byte aligned");
    return decode_impl(cfg, a, workspace, workspace_bytes, nullptr, mla::PartOut{nullptr, packed, num_slices, nullptr, 0},
                       reinterpret_cast<cudaStream_t>(stream));
}

mla_status_t mla_combine_partials_packed(const mla_config_t* cfg, mla_dtype_t dtype, int batch, int num_parts,
                                         int heads, const float* packed, const void* W_UV, float* output,
                                         mla_stream_t stream) {
    mla_status_t st = validate_cfg(cfg);
    if (st != MLA_OK) return st;
    if (!packed) return fail(MLA_ERR_INVALID_ARGUMENT, "packed input is null");
    if (reinterpret_cast<uintptr_t>(packed) % 16 != 0) return fail(MLA_ERR_INVALID_ARGUMENT, "packed must be 16-byte aligned");
    const int row = cfg->kv_lora_rank + 4;
    return combine_impl(cfg, dtype, batch, num_parts, heads, packed, packed + 4, row, row, W_UV, output,
                        reinterpret_cast<cudaStream_t>(stream));
}

mla_status_t mla_cache_append(const mla_config_t* cfg, mla_dtype_t dtype, void* kv_cache, int64_t kv_row_stride,
                              int64_t kv_total_rows, int batch, const void* c_t, const void* k_rope,
                              const int64_t* kv_offsets, const int* page_table, int page_rows, int max_pages,
                              int* seq_lens, int max_seq_len, int* status, mla_stream_t stream) {
    mla_status_t st = validate_cfg(cfg);
    if (st != MLA_OK) return st;
    if (!kv_cache || !c_t || !k_rope || !seq_lens) return fail(MLA_ERR_INVALID_ARGUMENT, "null pointer");
    if (batch <= 0) return fail(MLA_ERR_INVALID_ARGUMENT, "batch must be positive, got %d", batch);
    if (max_seq_len <= 0) return fail(MLA_ERR_INVALID_ARGUMENT, "max_seq_len must be positive, got %d", max_seq_len);
    const int dc = cfg->kv_lora_rank, dR = cfg->qk_rope_head_dim;
    const int64_t stride = kv_row_stride ? kv_row_stride : (dc + dR);
    if (stride < dc + dR) return fail(MLA_ERR_INVALID_ARGUMENT, "kv_row_stride %lld < d_c + d_R", (long long)stride);
    if (kv_total_rows < 0) return fail(MLA_ERR_INVALID_ARGUMENT, "kv_total_rows must be >= 0");
    // as for mla_decode: rows addressed through offsets are checked against the cache's rows
    if (kv_offsets && kv_total_rows <= 0)
        return fail(MLA_ERR_INVALID_ARGUMENT, "kv_total_rows is required with kv_offsets");
    if (page_table) {
        if (kv_offsets) return fail(MLA_ERR_INVALID_ARGUMENT, "page_table excludes kv_offsets");
        if (page_rows <= 0) return fail(MLA_ERR_INVALID_ARGUMENT, "page_rows must be positive, got %d", page_rows);
        if (static_cast<long long>(max_pages) * page_rows < max_seq_len)
            return fail(MLA_ERR_INVALID_ARGUMENT, "max_pages %d x page_rows %d < max_seq_len %d", max_pages, page_rows,
                        max_seq_len);
        if (kv_total_rows <= 0)
            return fail(MLA_ERR_INVALID_ARGUMENT, "kv_total_rows (rows of the page pool) is required with page_table");
    }
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    cudaError_t e;
    if (dtype == MLA_DTYPE_BF16)
        e = mla::launch_cache_append<__nv_bfloat16>(static_cast<__nv_bfloat16*>(kv_cache), stride, kv_total_rows, dc,
                                                    dR, batch, static_cast<const __nv_bfloat16*>(c_t),
                                                    static_cast<const __nv_bfloat16*>(k_rope), kv_offsets, page_table,
                                                    page_rows, max_pages, seq_lens, max_seq_len, status, s);
    else if (dtype == MLA_DTYPE_F16)
        e = mla::launch_cache_append<__half>(static_cast<__half*>(kv_cache), stride, kv_total_rows, dc, dR, batch,
                                             static_cast<const __half*>(c_t), static_cast<const __half*>(k_rope),
                                             kv_offsets, page_table, page_rows, max_pages, seq_lens, max_seq_len,
                                             status, s);
    else
        return fail(MLA_ERR_UNSUPPORTED, "dtype must be F16 or BF16");
    if (e == cudaErrorNoKernelImageForDevice || e == cudaErrorInvalidDeviceFunction)
        return fail(MLA_ERR_NO_DEVICE_CODE, "cache append kernel: %s (library is built for sm_100a)", cudaGetErrorString(e));
    if (e != cudaSuccess) return cuda_fail(e, "cache append kernel launch");
    return MLA_OK;
}

mla_status_t mla_launch_fused(const mla_fused_params_t* p, mla_dtype_t dtype, mla_stream_t stream) {
    if (!p) return fail(MLA_ERR_INVALID_ARGUMENT, "params is null");
    mla_status_t st = validate_cfg(p->cfg);
    if (st != MLA_OK) return st;
    if (!p->output) return fail(MLA_ERR_INVALID_ARGUMENT, "output is null");
    if (!p->q_absorbed) return fail(MLA_ERR_INVALID_ARGUMENT, "q_absorbed is null");
    if (p->seq_len <= 0) return fail(MLA_ERR_INVALID_ARGUMENT, "seq_len must be positive, got %d", p->seq_len);
    mla_decode_args_t a;
    std::memset(&a, 0, sizeof(a));
    a.dtype = dtype;
    a.batch = 1;
    a.kv_cache = p->kv_cache;
    a.max_seq_len = p->seq_len;
    a.q_absorbed = p->q_absorbed;
    a.q_rope = p->q_rope;
    a.W_UV = p->W_UV;
    a.rope_cos = p->rope_cos;
    a.rope_sin = p->rope_sin;
    a.output = p->output;
    return decode_with_pool(p->cfg, &a, reinterpret_cast<cudaStream_t>(stream));
}

mla_status_t mla_launch_batched_fused(const mla_batched_fused_params_t* p, mla_dtype_t dtype,
                                      mla_stream_t stream) {
    if (!p) return fail(MLA_ERR_INVALID_ARGUMENT, "params is null");
    mla_status_t st = validate_cfg(p->cfg);
    if (st != MLA_OK) return st;
    if (!p->output) return fail(MLA_ERR_INVALID_ARGUMENT, "output is null");
    if (!p->q_absorbed) return fail(MLA_ERR_INVALID_ARGUMENT, "q_absorbed is null");
    if (p->seq_len <= 0) return fail(MLA_ERR_INVALID_ARGUMENT, "seq_len must be positive, got %d", p->seq_len);
    if (p->batch_size <= 0) return fail(MLA_ERR_INVALID_ARGUMENT, "batch_size must be positive, got %d", p->batch_size);
    mla_decode_args_t a;
    std::memset(&a, 0, sizeof(a));
    a.dtype = dtype;
    a.batch = p->batch_size;
    a.shared_cache = 1;
    a.kv_cache = p->kv_cache;
    a.max_seq_len = p->seq_len;
    a.q_absorbed = p->q_absorbed;
    a.q_rope = p->q_rope;
    a.W_UV = p->W_UV;
    a.rope_cos = p->rope_cos;
    a.rope_sin = p->rope_sin;
    a.output = p->output;
    return decode_with_pool(p->cfg, &a, reinterpret_cast<cudaStream_t>(stream));
}

mla_status_t mla_timer_create(mla_timer_t* timer) {
    if (!timer) return fail(MLA_ERR_INVALID_ARGUMENT, "timer is null");
    auto* t = new mla_timer_st();
    cudaError_t e = cudaEventCreate(&t->begin);
    if (e == cudaSuccess) e = cudaEventCreate(&t->end);
    if (e != cudaSuccess) {
        if (t->begin) cudaEventDestroy(t->begin);
        delete t;
        return cuda_fail(e, "cudaEventCreate");
    }
    *timer = t;
    return MLA_OK;
}

mla_status_t mla_timer_destroy(mla_timer_t timer) {
    if (!timer) return MLA_OK;
    cudaEventDestroy(timer->begin);
    cudaEventDestroy(timer->end);
    delete timer;
    return MLA_OK;
}

mla_status_t mla_timer_decode_ms(mla_timer_t timer, float* ms) {
    if (!timer || !ms) return fail(MLA_ERR_INVALID_ARGUMENT, "null argument");
    if (!timer->recorded) return fail(MLA_ERR_INVALID_ARGUMENT, "timer has not been used by a decode call");
    cudaError_t e = cudaEventSynchronize(timer->end);
    if (e == cudaSuccess) e = cudaEventElapsedTime(ms, timer->begin, timer->end);
    if (e != cudaSuccess) return cuda_fail(e, "timer");
    return MLA_OK;
}

uint64_t mla_kernel_launch_count(void) { return mla::g_launches.load(std::memory_order_relaxed); }

mla_status_t mla_launch_fused_noalloc(const mla_fused_params_t* p, mla_dtype_t dtype, mla_stream_t stream) {
    if (!p) return fail(MLA_ERR_INVALID_ARGUMENT, "params is null");
    mla_status_t st = validate_cfg(p->cfg);
    if (st != MLA_OK) return st;
    if (!p->output) return fail(MLA_ERR_INVALID_ARGUMENT, "output is null");
    if (!p->q_absorbed) return fail(MLA_ERR_INVALID_ARGUMENT, "q_absorbed is null");
    if (p->seq_len <= 0) return fail(MLA_ERR_INVALID_ARGUMENT, "seq_len must be positive, got %d", p->seq_len);
    mla_decode_args_t a;
    std::memset(&a, 0, sizeof(a));
    a.dtype = dtype;
    a.batch = 1;
    a.kv_cache = p->kv_cache;
    a.max_seq_len = p->seq_len;
    a.q_absorbed = p->q_absorbed;
    a.q_rope = p->q_rope;
    a.W_UV = p->W_UV;
    a.rope_cos = p->rope_cos;
    a.rope_sin = p->rope_sin;
    a.output = p->output;
    // Largest worker count whose workspace fits the static array (fewer workers, fewer
    // partial records). Each worker beyond the first adds one record of kGroupRows rows of
    // (m, l) fp32 and o[d_c] in the 16-bit cache type, each part a multiple of the 256-byte
    // alignment, so the scratch grows by
    // exactly that much per worker and the cap follows from the one-worker size. A problem
    // that does not fit even with one worker is rejected before anything is launched.
    Plan pl;
    st = make_plan(p->cfg, &a, &pl, 1);
    if (st != MLA_OK) return st;
    if (pl.total > MLA_NOALLOC_SCRATCH_BYTES)
        return fail(MLA_ERR_UNSUPPORTED,
                    "problem needs %zu bytes of scratch; the static scratch of mla_launch_fused_noalloc holds %u",
                    pl.total, static_cast<unsigned>(MLA_NOALLOC_SCRATCH_BYTES));
    const size_t per_worker =
        static_cast<size_t>(mla::kGroupRows) * (2 * sizeof(float) + static_cast<size_t>(p->cfg->kv_lora_rank) * 2);
    const size_t extra = (MLA_NOALLOC_SCRATCH_BYTES - pl.total) / per_worker;
    const int workers = static_cast<int>(extra > 4096 ? 4097 : extra + 1);
    st = make_plan(p->cfg, &a, &pl, workers);
    if (st != MLA_OK) return st;
    if (pl.total > MLA_NOALLOC_SCRATCH_BYTES)  // the per-worker step above is exact; kept as a guard
        return fail(MLA_ERR_UNSUPPORTED, "static scratch plan does not fit (%zu bytes)", pl.total);
    void* scratch = nullptr;
    st = noalloc_scratch(&scratch);
    if (st != MLA_OK) return st;
    return decode_impl(p->cfg, &a, scratch, MLA_NOALLOC_SCRATCH_BYTES, a.output, mla::PartOut{},
                       reinterpret_cast<cudaStream_t>(stream), workers);
}

mla_status_t mla_decode_partial_put(const mla_config_t* cfg, const mla_decode_args_t* a, int world, void* const* dst,
                                    size_t dst_offset, const mla_peer_signal_t* signal, void* workspace,
                                    size_t workspace_bytes, mla_stream_t stream) {
    mla_status_t st = validate_cfg(cfg);
    if (st != MLA_OK) return st;
    mla::PeerSig sig;
    st = peer_sig(signal, &sig);
    if (st != MLA_OK) return st;
    if (!dst) return fail(MLA_ERR_INVALID_ARGUMENT, "dst is null");
    if (world <= 0 || cfg->num_heads % world != 0)
        return fail(MLA_ERR_INVALID_ARGUMENT, "world (%d) must divide num_heads (%d)", world, cfg->num_heads);
    if (dst_offset % 16 != 0) return fail(MLA_ERR_INVALID_ARGUMENT, "dst_offset must be a multiple of 16 bytes");
    return decode_impl(cfg, a, workspace, workspace_bytes, nullptr, mla::PartOut{nullptr, nullptr, world, dst, dst_offset},
                       reinterpret_cast<cudaStream_t>(stream), 0, sig);
}

mla_status_t mla_combine_partials_put(const mla_config_t* cfg, mla_dtype_t dtype, int batch, int num_parts, int heads,
                                      const float* packed, const void* W_UV, int world, void* const* dst,
                                      size_t dst_offset, size_t dst_pitch, const mla_peer_signal_t* signal,
                                      float* scratch, mla_stream_t stream) {
    mla_status_t st = validate_cfg(cfg);
    if (st != MLA_OK) return st;
    mla::PeerSig sig;
    st = peer_sig(signal, &sig);
    if (st != MLA_OK) return st;
    if (!packed || !dst || !scratch) return fail(MLA_ERR_INVALID_ARGUMENT, "null pointer");
    if (world <= 0 || world > 512) return fail(MLA_ERR_INVALID_ARGUMENT, "world must be in [1, 512]");
    if (reinterpret_cast<uintptr_t>(packed) % 16 != 0 || reinterpret_cast<uintptr_t>(scratch) % 16 != 0)
        return fail(MLA_ERR_INVALID_ARGUMENT, "packed and scratch must be 16-byte aligned");
    if (dst_offset % 16 != 0 || dst_pitch % 16 != 0)
        return fail(MLA_ERR_INVALID_ARGUMENT, "dst_offset and dst_pitch must be multiples of 16 bytes");
    if (heads > 0 && dst_pitch < static_cast<size_t>(heads) * cfg->v_head_dim * sizeof(float))
        return fail(MLA_ERR_INVALID_ARGUMENT, "dst_pitch is shorter than a token's rows");
    const int row = cfg->kv_lora_rank + 4;
    const mla::PeerRows rows{dst, dst_offset, dst_pitch, world, sig};
    return combine_impl(cfg, dtype, batch, num_parts, heads, packed, packed + 4, row, row, W_UV, scratch,
                        reinterpret_cast<cudaStream_t>(stream), rows);
}

mla_status_t mla_decode_partial_gather(const mla_config_t* cfg, const mla_decode_args_t* a, int world, void* const* dst,
                                       size_t dst_offset, size_t parity_bytes, const mla_peer_signal_t* signal,
                                       void* workspace, size_t workspace_bytes, mla_stream_t stream) {
    mla_status_t st = validate_cfg(cfg);
    if (st != MLA_OK) return st;
    mla::PeerSig sig;
    st = peer_sig(signal, &sig);
    if (st != MLA_OK) return st;
    if (!a) return fail(MLA_ERR_INVALID_ARGUMENT, "args is null");
    if (!dst) return fail(MLA_ERR_INVALID_ARGUMENT, "dst is null");
    if (world <= 0 || world > 512) return fail(MLA_ERR_INVALID_ARGUMENT, "world must be in [1, 512]");
    if (a->batch < 1 || a->batch > 4) return fail(MLA_ERR_UNSUPPORTED, "the gathered export takes batch 1 .. 4");
    if (dst_offset % 16 != 0 || parity_bytes % 16 != 0)
        return fail(MLA_ERR_INVALID_ARGUMENT, "dst_offset and parity_bytes must be multiples of 16 bytes");
    mla::PartOut part{nullptr, nullptr, 0, dst, dst_offset, world, parity_bytes};
    return decode_impl(cfg, a, workspace, workspace_bytes, nullptr, part, reinterpret_cast<cudaStream_t>(stream), 0, sig);
}

mla_status_t mla_combine_partials_gathered(const mla_config_t* cfg, mla_dtype_t dtype, int batch, int num_parts,
                                           const float* packed, size_t parity_bytes, const int* epoch, const void* W_UV,
                                           float* output, mla_stream_t stream) {
    mla_status_t st = validate_cfg(cfg);
    if (st != MLA_OK) return st;
    if (!packed || !epoch) return fail(MLA_ERR_INVALID_ARGUMENT, "packed and epoch must be non-null");
    if (reinterpret_cast<uintptr_t>(packed) % 16 != 0 || parity_bytes % 16 != 0)
        return fail(MLA_ERR_INVALID_ARGUMENT, "packed and parity_bytes must be 16-byte aligned");
    const int row = cfg->kv_lora_rank + 4;
    return combine_impl(cfg, dtype, batch, num_parts, cfg->num_heads, packed, packed + 4, row, row, W_UV, output,
                        reinterpret_cast<cudaStream_t>(stream), mla::PeerRows{}, epoch, parity_bytes / sizeof(float));
}

mla_status_t mla_decode_kv_range(const mla_config_t* cfg, const mla_decode_args_t* a, int world, int rank,
                                 void* const* recv, size_t half_bytes, int* epoch, unsigned int* counter, int* status,
                                 void* workspace, size_t workspace_bytes, mla_stream_t stream) {
    mla_status_t st = validate_cfg(cfg);
    if (st != MLA_OK) return st;
    if (!a) return fail(MLA_ERR_INVALID_ARGUMENT, "args is null");
    if (!a->output) return fail(MLA_ERR_INVALID_ARGUMENT, "output is null");
    if (!recv || !epoch || !counter || !status)
        return fail(MLA_ERR_INVALID_ARGUMENT, "recv, epoch, counter and status must be non-null");
    if (world < 1 || world > 64 || rank < 0 || rank >= world)
        return fail(MLA_ERR_INVALID_ARGUMENT, "world must be in [1, 64] and rank in [0, world)");
    if (a->batch < 1 || a->batch > 4) return fail(MLA_ERR_UNSUPPORTED, "the KV-range exchange takes batch 1 .. 4");
    if (cfg->v_head_dim != 128 || cfg->kv_lora_rank % 64 != 0 || cfg->kv_lora_rank > 512)
        return fail(MLA_ERR_UNSUPPORTED, "the KV-range exchange needs v_head_dim 128 and kv_lora_rank a multiple of 64 "
                                         "up to 512");
    const size_t need = static_cast<size_t>(world) * a->batch * cfg->num_heads * (cfg->kv_lora_rank + 4) * 8;
    if (half_bytes % 16 != 0 || half_bytes < need)
        return fail(MLA_ERR_INVALID_ARGUMENT, "half_bytes must be a multiple of 16 and at least %zu", need);
    const mla::LLRing ring{recv, half_bytes, world, rank, epoch, counter, status};
    return decode_impl(cfg, a, workspace, workspace_bytes, a->output, mla::PartOut{},
                       reinterpret_cast<cudaStream_t>(stream), 0, mla::PeerSig{}, &ring);
}

mla_status_t mla_ipc_alloc(size_t bytes, void** ptr, void* handle) {
    if (!ptr || !handle) return fail(MLA_ERR_INVALID_ARGUMENT, "null pointer");
    if (bytes == 0) return fail(MLA_ERR_INVALID_ARGUMENT, "bytes must be positive");
    *ptr = nullptr;
    const cudaError_t e = mla::ipc_alloc(bytes, ptr, handle);
    if (e != cudaSuccess) {
        if (*ptr) cudaFree(*ptr);
        *ptr = nullptr;
        return cuda_fail(e, "IPC allocation");
    }
    return MLA_OK;
}

mla_status_t mla_ipc_free(void* ptr) {
    if (!ptr) return MLA_OK;
    const cudaError_t e = cudaFree(ptr);
    return e == cudaSuccess ? MLA_OK : cuda_fail(e, "cudaFree");
}

mla_status_t mla_ipc_open(const void* handle, void** ptr) {
    if (!ptr || !handle) return fail(MLA_ERR_INVALID_ARGUMENT, "null pointer");
    const cudaError_t e = mla::ipc_open(handle, ptr);
    return e == cudaSuccess ? MLA_OK : cuda_fail(e, "cudaIpcOpenMemHandle");
}

mla_status_t mla_ipc_close(void* ptr) {
    if (!ptr) return MLA_OK;
    const cudaError_t e = cudaIpcCloseMemHandle(ptr);
    return e == cudaSuccess ? MLA_OK : cuda_fail(e, "cudaIpcCloseMemHandle");
}

mla_status_t mla_peer_put(const void* src, size_t rows, size_t row_bytes, size_t src_pitch, size_t src_stride,
                          void* const* dst, size_t dst_pitch, size_t dst_offset, int world, int blocks,
                          const mla_peer_signal_t* signal, mla_stream_t stream) {
    mla::PeerSig sig;
    mla_status_t st = peer_sig(signal, &sig);
    if (st != MLA_OK) return st;
    if (!src || !dst) return fail(MLA_ERR_INVALID_ARGUMENT, "null pointer");
    if (world <= 0 || world > 65535 || blocks <= 0 || blocks > 1024)
        return fail(MLA_ERR_INVALID_ARGUMENT, "world in [1, 65535], blocks in [1, 1024]");
    if (row_bytes % 16 || src_pitch % 16 || src_stride % 16 || dst_pitch % 16 || dst_offset % 16 ||
        reinterpret_cast<uintptr_t>(src) % 16)
        return fail(MLA_ERR_INVALID_ARGUMENT, "sizes, pitches, strides, offsets and src must be multiples of 16 bytes");
    if (rows == 0 || row_bytes == 0 || rows * (row_bytes / 16) >= (size_t{1} << 31) ||
        rows * src_pitch >= (size_t{1} << 32) || rows * dst_pitch >= (size_t{1} << 32))
        return fail(MLA_ERR_INVALID_ARGUMENT, "slice must be non-empty and span less than 4 GiB");
    const cudaError_t e = mla::launch_peer_put(src, rows, row_bytes, src_pitch, src_stride, dst, dst_pitch, dst_offset,
                                               world, blocks, sig, reinterpret_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? MLA_OK : cuda_fail(e, "peer put kernel launch");
}

mla_status_t mla_peer_wait(const int* flags, int count, int* epoch, int advance, int* status, mla_stream_t stream) {
    if (!flags || !epoch || count <= 0)
        return fail(MLA_ERR_INVALID_ARGUMENT, "flags and epoch must be non-null, count positive");
    const cudaError_t e =
        mla::launch_peer_wait(flags, count, epoch, advance, status, reinterpret_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? MLA_OK : cuda_fail(e, "peer wait kernel launch");
}

const char* mla_last_error(void) { return g_last_error.c_str(); }

const char* mla_version(void) { return "latent-attn-b200 0.1 (sm_100a)"; }

}  // extern "C"
