/*
 * latent-attn-b200 -- C ABI of the B200 (sm_100a) MLA decode library.
 *
 * Every entry point takes plain pointers and sizes, returns an mla_status_t,
 * never exits or aborts, never synchronises the host, and is asynchronous on
 * the given stream. Pointers are device pointers unless a name ends in _host.
 *
 * Entry points and the reference interface each one replaces
 * (anishesg/latent-attn, paths relative to that project):
 *
 *   mla_launch_fused          launch_fused_mla(const FusedMLAParams&, cudaStream_t)
 *                             src/fused_mla.cuh:11-34 (params), :51 (function)
 *   mla_launch_batched_fused  launch_batched_fused_mla(const BatchedFusedMLAParams&, cudaStream_t)
 *                             src/fused_mla_batched.cuh:7-30 (params), :35 (function)
 *   mla_decode                no reference counterpart: the general decode
 *                             (absorption in-op, variable-length batch, split-KV,
 *                             caller-provided workspace); it generalises the two
 *                             launchers above and the caller-side absorption of
 *                             tests/test_python.py:98-99
 *   mla_decode_partial /      no reference counterpart: the two halves of the
 *   mla_combine_partials      KV-range-sharded multi-GPU decode (per-head partial
 *   (and their _packed forms) (m, l, o_latent) out of one shard; log-sum-exp merge of
 *                             G shards' partials + the W_UV projection of
 *                             src/fused_mla.cu:258-267)
 *   mla_linear                the torch matmuls of LatentAttentionLayer.forward
 *                             (latent_attn/__init__.py:126, :128, :145)
 *   mla_cache_append          LatentKVCache::append_host (src/mla_config.cuh:58-72),
 *                             moved to the device for a whole batch
 *   mla_config_validate       MLAConfig::validate() (src/mla_config.cuh:35-40)
 */
#ifndef LATENT_ATTN_B200_MLA_H_
#define LATENT_ATTN_B200_MLA_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define MLA_API __attribute__((visibility("default")))
#else
#define MLA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Opaque stream handle, ABI-identical to cudaStream_t. */
typedef struct CUstream_st* mla_stream_t;

/* Opaque kernel timer (see mla_timer_create). */
typedef struct mla_timer_st* mla_timer_t;

typedef enum mla_status {
  MLA_OK = 0,
  MLA_ERR_INVALID_ARGUMENT = 1,   /* null pointer, bad size, non-positive dim */
  MLA_ERR_UNSUPPORTED = 2,        /* valid but not implemented (e.g. odd qk_rope_head_dim) */
  MLA_ERR_WORKSPACE = 3,          /* workspace pointer null / too small / misaligned */
  MLA_ERR_CUDA = 4,               /* a CUDA runtime call failed; see mla_last_error() */
  MLA_ERR_NO_DEVICE_CODE = 5,     /* the library was not built for this GPU (needs sm_100a) */
  MLA_ERR_TIMEOUT = 6             /* a device-side wait gave up (reported by the kernel) */
} mla_status_t;

typedef enum mla_dtype {
  MLA_DTYPE_F16 = 0,
  MLA_DTYPE_BF16 = 1,
  MLA_DTYPE_F32 = 2
} mla_dtype_t;

/* Same field order and types as MLAConfig (src/mla_config.cuh:7-13). */
typedef struct mla_config {
  int d_model;            /* not used by the decode op */
  int kv_lora_rank;       /* d_c */
  int qk_nope_head_dim;   /* dn */
  int qk_rope_head_dim;   /* d_R, even */
  int num_heads;          /* H */
  int v_head_dim;         /* dv */
} mla_config_t;

/* MLAConfig::validate(): MLA_ERR_INVALID_ARGUMENT when a dimension is not positive. */
MLA_API mla_status_t mla_config_validate(const mla_config_t* cfg);

/* Field order of FusedMLAParams (src/fused_mla.cuh:11-34). Element type of
 * kv_cache / W_UV is given by `dtype` (the reference is fp16-only). */
typedef struct mla_fused_params {
  const void* kv_cache;      /* (seq_len, d_c + d_R) packed [c_t | k_rope] */
  int seq_len;
  const float* q_absorbed;   /* (H, d_c) fp32 */
  const float* q_rope;       /* (H, d_R) fp32 */
  const void* W_UV;          /* (H * dv, d_c) */
  const float* rope_cos;     /* (seq_len, d_R / 2) fp32 */
  const float* rope_sin;     /* (seq_len, d_R / 2) fp32 */
  float* output;             /* (H, dv) fp32 */
  const mla_config_t* cfg;   /* read during the call only */
} mla_fused_params_t;

/* Field order of BatchedFusedMLAParams (src/fused_mla_batched.cuh:7-30):
 * batch_size query tokens attend to ONE shared cache. */
typedef struct mla_batched_fused_params {
  const void* kv_cache;      /* (seq_len, d_c + d_R) */
  int seq_len;
  int batch_size;
  const float* q_absorbed;   /* (B, H, d_c) fp32 */
  const float* q_rope;       /* (B, H, d_R) fp32 */
  const void* W_UV;          /* (H * dv, d_c) */
  const float* rope_cos;     /* (seq_len, d_R / 2) fp32 */
  const float* rope_sin;
  float* output;             /* (B, H, dv) fp32 */
  const mla_config_t* cfg;
} mla_batched_fused_params_t;

/* Drop-in for launch_fused_mla. The reference signature has no workspace, so the
 * split-KV scratch is taken stream-ordered from the device's default memory
 * pool (cudaMallocAsync / cudaFreeAsync on `stream`). */
MLA_API mla_status_t mla_launch_fused(const mla_fused_params_t* p, mla_dtype_t dtype, mla_stream_t stream);

/* Drop-in for launch_batched_fused_mla (same scratch policy). */
MLA_API mla_status_t mla_launch_batched_fused(const mla_batched_fused_params_t* p, mla_dtype_t dtype,
                                      mla_stream_t stream);

/* Allocation-free variant of mla_launch_fused. No counterpart in the reference.
 *
 * Some callers may not allocate device memory at all: hosts that own every
 * device allocation themselves (plugin and inference-server runtimes with a
 * pre-reserved arena), and latency-critical loops where an allocator call (and
 * the synchronisation it can imply) is not acceptable. mla_launch_fused takes
 * its split-KV scratch from the stream-ordered pool; this entry point instead
 * uses one fixed array of MLA_NOALLOC_SCRATCH_BYTES that the library keeps in
 * device memory on every GPU that loads it, until the process exits. It calls no
 * cudaMalloc, cudaMallocAsync, cudaFree or other allocating routine.
 *
 * - The caller still provides all inputs and the output, as for mla_launch_fused.
 * - Problems whose scratch does not fit (many heads or a large d_c) are
 *   rejected with MLA_ERR_UNSUPPORTED before anything runs; the split-KV worker
 *   count is reduced until the partial records fit.
 * - The first call on a device looks up the array's device address
 *   (cudaGetSymbolAddress) with that device current; make that first call
 *   before capturing any stream.
 * - Every call uses the same array: calls that can overlap on the GPU (other
 *   streams, other host threads) race and corrupt each other's results; order
 *   them on one stream. */
#define MLA_NOALLOC_SCRATCH_BYTES (8u << 20)
MLA_API mla_status_t mla_launch_fused_noalloc(const mla_fused_params_t* p, mla_dtype_t dtype, mla_stream_t stream);

/* General decode. One query token per sequence (or, with shared_cache, `batch`
 * tokens over sequence 0). */
typedef struct mla_decode_args {
  mla_dtype_t dtype;            /* element type of kv_cache, W_UK, W_UV: F16 or BF16 */
  int batch;                    /* B >= 1 */
  int shared_cache;             /* nonzero: all B tokens attend to the same rows (reference batched op) */
  const void* kv_cache;         /* packed rows [c_t | k_rope] */
  int64_t kv_row_stride;        /* elements between rows; 0 means d_c + d_R */
  int64_t kv_total_rows;        /* rows addressable from kv_cache (reads never go past them);
                                   0: max_seq_len if shared_cache or kv_offsets is NULL and B == 1,
                                   else batch * max_seq_len when kv_offsets is NULL; required with kv_offsets */
  const int64_t* kv_offsets;    /* device (B,) first row of sequence b; NULL: b * max_seq_len (0 if shared) */
  const int* seq_lens;          /* device (B,) positions per sequence; NULL: every sequence has max_seq_len */
  const int* seq_lens_host;     /* optional host copy of seq_lens (lets the planner skip a device scan) */
  int max_seq_len;              /* upper bound of seq_lens (>= 1) */
  int kv_pos_offset;            /* RoPE table row of cache row 0 (KV-range shards); usually 0 */
  /* queries: q_absorbed, or q_nope together with W_UK (absorption runs in-op) */
  const float* q_absorbed;      /* (B, H, d_c) fp32, or NULL */
  const float* q_nope;          /* (B, H, dn) fp32, or NULL */
  const void* W_UK;             /* (H * dn, d_c), required with q_nope */
  const float* q_rope;          /* (B, H, d_R) fp32, already rotated to the query position */
  const void* W_UV;             /* (H * dv, d_c) */
  const float* rope_cos;        /* (kv_pos_offset + max_seq_len, d_R/2) fp32, or NULL (see rope_theta) */
  const float* rope_sin;
  float softmax_scale;          /* 0: 1 / sqrt(dn + d_R) */
  float* output;                /* (B, H, dv) fp32 */
  int kernel;                   /* MLA_KERNEL_AUTO (0), MLA_KERNEL_TENSOR_CORE (1), MLA_KERNEL_CUDA_CORE (2) */
  mla_timer_t timer;            /* optional: CUDA events are recorded around the decode kernel */
  /* Paged cache (block table), optional. With page_table, position p of sequence b is row
   * page_table[b * max_pages + p / page_rows] * page_rows + p % page_rows of kv_cache, and
   * kv_total_rows (the page pool's rows) is required; kv_offsets and shared_cache must be unset.
   * A page id outside the pool reads no memory: the tile reads as zeros, the status word
   * records the error and the output becomes NaN. */
  const int* page_table;        /* device (B, max_pages) int32 page ids, or NULL (contiguous layout) */
  int page_rows;                /* rows per page, a positive multiple of 64 */
  int max_pages;                /* page-table entries per sequence, >= ceil(max_seq_len / page_rows) */
  /* On-the-fly RoPE. With rope_cos and rope_sin both NULL the decode kernels compute the
   * rotation of each cache row themselves, with the reference table builder's rotate-half
   * convention (latent_attn/__init__.py:31-38): freq_i = rope_theta^(-2i / d_R) (a
   * double-precision power rounded to fp32) and angle = pos * freq_i taken exactly (the table
   * builder rounds it to fp32, a difference of at most half an fp32 ulp of the angle); cos / sin
   * are within 6e-7 of their exact values. No table is read. 0 means 10000. Ignored when tables
   * are given; needs qk_rope_head_dim <= 128 and positions below 2^29. */
  float rope_theta;
} mla_decode_args_t;

enum { MLA_KERNEL_AUTO = 0, MLA_KERNEL_TENSOR_CORE = 1, MLA_KERNEL_CUDA_CORE = 2 };

/* Bytes of workspace mla_decode needs for these arguments (256-byte aligned). */
MLA_API mla_status_t mla_decode_workspace_size(const mla_config_t* cfg, const mla_decode_args_t* a,
                                       size_t* bytes);

MLA_API mla_status_t mla_decode(const mla_config_t* cfg, const mla_decode_args_t* a, void* workspace,
                        size_t workspace_bytes, mla_stream_t stream);

/* KV-range sharding, step 1: decode over this rank's rows only and write one
 * partial per (b, h): m (natural-log units), l, and the UNnormalised latent sum
 * o (d_c floats). partial_ml: (B, H, 2) fp32; partial_o: (B, H, d_c) fp32.
 * Uses the same workspace as mla_decode (mla_decode_workspace_size). */
MLA_API mla_status_t mla_decode_partial(const mla_config_t* cfg, const mla_decode_args_t* a,
                                float* partial_ml, float* partial_o, void* workspace,
                                size_t workspace_bytes, mla_stream_t stream);

/* KV-range sharding, step 2: merge `num_parts` partial sets laid out
 * (num_parts, B, H, .) and project through W_UV: output (B, H, dv) fp32. */
MLA_API mla_status_t mla_combine_partials(const mla_config_t* cfg, mla_dtype_t dtype, int batch,
                                  int num_parts, const float* partial_ml, const float* partial_o,
                                  const void* W_UV, float* output, mla_stream_t stream);

/* KV-range sharding with a head-sliced exchange, step 1: as mla_decode_partial, but every
 * (b, h) partial is one packed row of d_c + 4 floats [m (natural-log units), l, 0, 0,
 * o[0 .. d_c)], and the rows are ordered by head slice: the heads are cut into num_slices
 * equal slices (num_slices divides H; slice q holds heads [q H / num_slices, + H / num_slices)),
 * and head h of token b is row (q * B + b) * (H / num_slices) + h % (H / num_slices). Slice q is
 * thus one contiguous block, ready for an all-to-all that sends it to the rank merging those
 * heads. packed: (num_slices, B, H / num_slices, d_c + 4) fp32, 16-byte aligned. No reference
 * counterpart (the reference has no multi-GPU path). */
MLA_API mla_status_t mla_decode_partial_packed(const mla_config_t* cfg, const mla_decode_args_t* a, int num_slices,
                                       float* packed, void* workspace, size_t workspace_bytes,
                                       mla_stream_t stream);

/* KV-range sharding with a head-sliced exchange, step 2: merge num_parts packed partial sets
 * (num_parts, B, heads, d_c + 4) of one head slice (the rows of mla_decode_partial_packed that
 * all ranks sent for it) and project through that slice's W_UV rows (heads * dv, d_c): output
 * (B, heads, dv) fp32. The log-sum-exp merge of mla_combine_partials and the projection of
 * src/fused_mla.cu:258-267, for a subset of the heads. */
MLA_API mla_status_t mla_combine_partials_packed(const mla_config_t* cfg, mla_dtype_t dtype, int batch,
                                         int num_parts, int heads, const float* packed, const void* W_UV,
                                         float* output, mla_stream_t stream);

/* Projection GEMM for the layer-level caller: Y (M, N) fp32 = X (M, K) . W (N, K)^T, with X and W
 * row-major fp16 or bf16 (both `dtype`), 1 <= M <= 256 tokens, K a multiple of 8. It replaces the
 * torch matmuls of the reference's LatentAttentionLayer.forward (latent_attn/__init__.py:126,
 * :128, :145: x @ W_Q_absorbed^T, x @ W_Q_rope^T and the W_O projection); no counterpart in the
 * reference's kernels. Weight-streaming tcgen05 kernel: every weight byte is read once for all M
 * tokens. When N is small for the GPU the K range is split over CTAs that add into Y (the call
 * zeroes Y first, on the stream), so results can differ in the last bits from run to run. */
MLA_API mla_status_t mla_linear(mla_dtype_t dtype, int M, int N, int K, const void* X, const void* W, float* Y,
                                mla_stream_t stream);

/* ---- Peer memory for the multi-GPU exchange (one process per GPU, GPUs of one node) ----
 * The KV-range decode's two exchanges (per-head partials to the rank that merges those heads,
 * then the merged outputs to every rank) can run as direct NVLink stores into the peers'
 * buffers instead of NCCL collectives: no reference counterpart (the reference is single-GPU). */
#define MLA_IPC_HANDLE_BYTES 64

/* Allocates `bytes` of device memory on the current device that other processes can map:
 * *ptr receives the local pointer and handle (MLA_IPC_HANDLE_BYTES bytes) the handle to pass
 * to the peers (cudaIpcGetMemHandle). Free with mla_ipc_free. */
MLA_API mla_status_t mla_ipc_alloc(size_t bytes, void** ptr, void* handle);
MLA_API mla_status_t mla_ipc_free(void* ptr);
/* Maps a peer's allocation from its handle (cudaIpcOpenMemHandle with lazy peer access);
 * unmap with mla_ipc_close. */
MLA_API mla_status_t mla_ipc_open(const void* handle, void** ptr);
MLA_API mla_status_t mla_ipc_close(void* ptr);

/* How a kernel that stores into other ranks' buffers tells them its data has landed. Receiver q
 * has an int flag word per sender; this rank sets word `flag_index` of every receiver to
 * *epoch + 1 once the kernel's stores bound for q are complete (system-scope release). The
 * kernel's blocks count themselves per receiver in `counters` (world zeroed words of THIS rank's
 * device memory, left zeroed); the block that completes a count releases the flag. flags and
 * counters are DEVICE arrays (world pointers; world words); epoch is a device int of this rank. */
typedef struct mla_peer_signal {
    int* const* flags;
    int flag_index;
    const int* epoch;
    unsigned int* counters;
} mla_peer_signal_t;

/* One kernel: for q < world, copies slice q of src to dst[q] and then signals receiver q. Slice
 * q is `rows` rows of row_bytes; row i starts at src + q * src_stride + i * src_pitch and lands at
 * dst[q] + dst_offset + i * dst_pitch (src_stride 0 sends the same slice to every rank: an
 * all-gather; distinct slices make one rank's side of an all-to-all). Every size, pitch, stride,
 * offset and pointer is a multiple of 16 bytes. `blocks` thread blocks share each slice. dst is
 * a DEVICE array of `world` pointers (peer memory from mla_ipc_open, or local memory). */
MLA_API mla_status_t mla_peer_put(const void* src, size_t rows, size_t row_bytes, size_t src_pitch, size_t src_stride,
                                  void* const* dst, size_t dst_pitch, size_t dst_offset, int world, int blocks,
                                  const mla_peer_signal_t* signal, mla_stream_t stream);
/* mla_decode_partial_packed with its packed rows stored straight into the ranks that merge them:
 * slice q (the B * H / world rows of heads [q H / world, (q + 1) H / world), ordered (token,
 * head within the slice)) lands at dst[q] + dst_offset, and receiver q is signalled once it has
 * (see mla_peer_signal_t). The export kernel itself does the stores (over NVLink for peers): one
 * kernel replaces the export and the sender's half of an all-to-all. world divides num_heads;
 * dst is a DEVICE array of world pointers; dst_offset a multiple of 16. */
MLA_API mla_status_t mla_decode_partial_put(const mla_config_t* cfg, const mla_decode_args_t* args, int world,
                                            void* const* dst, size_t dst_offset, const mla_peer_signal_t* signal,
                                            void* workspace, size_t workspace_bytes, mla_stream_t stream);
/* mla_combine_partials_packed with the (batch, heads, dv) fp32 output stored into every rank:
 * token b's rows land at dst[q] + dst_offset + b * dst_pitch for every q < world, then every
 * receiver is signalled. For batch <= 4 the merge kernel does the stores; larger batches are
 * staged in scratch (batch * heads * dv floats of this rank) and sent by a put kernel. One call
 * is this rank's half of the output all-gather. */
MLA_API mla_status_t mla_combine_partials_put(const mla_config_t* cfg, mla_dtype_t dtype, int batch, int num_parts,
                                              int heads, const float* packed, const void* W_UV_slice, int world,
                                              void* const* dst, size_t dst_offset, size_t dst_pitch,
                                              const mla_peer_signal_t* signal, float* scratch, mla_stream_t stream);
/* The gathered exchange for small batches (batch 1 .. 4, the long-sequence case): every rank
 * receives every rank's partials of all heads and merges them itself, so one exchange replaces the
 * all-to-all and the output all-gather. mla_decode_partial_gather stores this rank's (batch, H)
 * packed rows [m, l, 0, 0, o] (rows ordered (token, head), kv_lora_rank + 4 floats each) at
 * dst[q] + dst_offset + ((*epoch + 1) & 1) * parity_bytes for every q < world, then signals every
 * receiver: the receive area is double-buffered by the step's flag value, so a rank may run one
 * step ahead of a slower peer without overwriting what that peer is still merging.
 * mla_combine_partials_gathered merges num_parts sets (num_parts, batch, H, kv_lora_rank + 4) at
 * packed + (*epoch & 1) * parity_bytes (after mla_peer_wait with advance has moved *epoch to the
 * step's flag value) and projects with W_UV into output (batch, H, v_head_dim) fp32. */
MLA_API mla_status_t mla_decode_partial_gather(const mla_config_t* cfg, const mla_decode_args_t* args, int world,
                                               void* const* dst, size_t dst_offset, size_t parity_bytes,
                                               const mla_peer_signal_t* signal, void* workspace,
                                               size_t workspace_bytes, mla_stream_t stream);
MLA_API mla_status_t mla_combine_partials_gathered(const mla_config_t* cfg, mla_dtype_t dtype, int batch,
                                                   int num_parts, const float* packed, size_t parity_bytes,
                                                   const int* epoch, const void* W_UV, float* output,
                                                   mla_stream_t stream);
/* One rank's whole KV-range decode step for batch 1 .. 4, with the exchange inside one kernel:
 * absorption, the decode of this rank's rows (args as for mla_decode, kv_pos_offset = the rows'
 * first position, output (batch, H, v_head_dim) fp32 on this rank), then a kernel whose block h
 * merges the rank's split-KV records of head h, stores the packed partial into every other rank's
 * receive area (NVLink stores), reads every other rank's partial of head h from its own area, merges
 * the world partials in rank order and projects them with W_UV. Each 16-byte store carries two
 * values and the step number (*epoch + 1) beside each, so a reader waits (bounded, 2 s) on the data
 * itself: no flag, no fence, no separate wait kernel.
 * - recv: DEVICE array of world pointers to every rank's receive area (this rank's included),
 *   2 x half_bytes each, zeroed once at setup; half_bytes >= world * batch * H * (kv_lora_rank + 4)
 *   * 8, a multiple of 16. The two halves alternate by step, so a rank one step ahead never
 *   overwrites rows a slower peer is still reading.
 * - epoch, counter, status: device ints of this rank, zeroed at setup. The kernel advances *epoch
 *   once per call; every rank must make the same sequence of calls. A wait that gives up sets
 *   *status to 1 and that head's output to NaN. */
MLA_API mla_status_t mla_decode_kv_range(const mla_config_t* cfg, const mla_decode_args_t* args, int world, int rank,
                                         void* const* recv, size_t half_bytes, int* epoch, unsigned int* counter,
                                         int* status, void* workspace, size_t workspace_bytes, mla_stream_t stream);
/* Waits on the device (one small kernel, bounded: 2 s) until flags[i] >= *epoch + 1 for i < count,
 * with system-scope acquire ordering, so the kernels after it on the stream see the data the
 * peers stored before their flags; with advance != 0 it then increments *epoch (the last wait of
 * an exchange step), so that a captured CUDA graph replays with a new value each time. A wait
 * that gives up stores 1 to *status (a device int, or NULL) and leaves *epoch unchanged. */
MLA_API mla_status_t mla_peer_wait(const int* flags, int count, int* epoch, int advance, int* status,
                                   mla_stream_t stream);

/* Device-side cache append, one new row per sequence: for each b, the row of position
 * p = seq_lens[b] receives [c_t[b] (d_c) | k_rope[b] (d_R)] (k_rope unrotated, as the cache
 * stores it) and seq_lens[b] advances by one. The row is (kv_offsets ? kv_offsets[b] :
 * b * max_seq_len) + p, or, with page_table, page_table[b * max_pages + p / page_rows] *
 * page_rows + p % page_rows (the layout mla_decode reads with the same table). Everything
 * happens on the stream: no host copy, no synchronisation, so a decode step can append and
 * attend without the host.
 * Replaces LatentKVCache::append_host (src/mla_config.cuh:58-72), which copies one
 * position from host memory and synchronises the stream per token.
 * - c_t (batch, d_c) and k_rope (batch, d_R): device, element type `dtype`.
 * - seq_lens (batch,) int32 device, read and advanced; kv_offsets (batch,) int64 device or
 *   NULL; page_table (batch, max_pages) int32 device or NULL (page_rows > 0 with it).
 * - kv_total_rows: rows of kv_cache; required with page_table or kv_offsets (a row outside
 *   it is not written), 0 allowed only without both.
 * - A sequence that already holds max_seq_len rows is left unchanged and sets bit 0 of
 *   *status; a row outside the cache (a bad page id or offset) is not written and sets
 *   bit 1 (status: a device int, or NULL).
 * - kv_row_stride: elements between rows, 0 meaning d_c + d_R. */
MLA_API mla_status_t mla_cache_append(const mla_config_t* cfg, mla_dtype_t dtype, void* kv_cache,
                              int64_t kv_row_stride, int64_t kv_total_rows, int batch, const void* c_t,
                              const void* k_rope, const int64_t* kv_offsets, const int* page_table,
                              int page_rows, int max_pages, int* seq_lens, int max_seq_len, int* status,
                              mla_stream_t stream);

/* Kernel timing for benchmarks: a timer passed in mla_decode_args_t.timer gets
 * CUDA events recorded on the call's stream immediately before and after the
 * split-KV decode kernel. mla_timer_decode_ms waits for the second event and
 * returns the elapsed milliseconds of the most recent such call. */
MLA_API mla_status_t mla_timer_create(mla_timer_t* timer);
MLA_API mla_status_t mla_timer_destroy(mla_timer_t timer);
MLA_API mla_status_t mla_timer_decode_ms(mla_timer_t timer, float* ms);

/* Number of CUDA kernels this library has launched in this process so far. */
MLA_API uint64_t mla_kernel_launch_count(void);

/* Thread-local message for the last non-OK status returned on this thread. */
MLA_API const char* mla_last_error(void);

/* Library build/version string. */
MLA_API const char* mla_version(void);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* LATENT_ATTN_B200_MLA_H_ */
