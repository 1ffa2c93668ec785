/*
 * tvb200 — B200-native (sm_100a) quantized-weight hot path for ternative.
 *
 * Plain C ABI: device pointers, host pointers and sizes only; no C++ or torch
 * types.  Every call returns a tvb_status and never throws.  A failed call
 * leaves a message readable with tvb_last_error() (per host thread).
 *
 * All device work is asynchronous on the stream passed in (`stream` is a
 * cudaStream_t; NULL = the legacy default stream), except where a function
 * says it synchronises.
 *
 * Reference interfaces replaced (paths inside the ternative project):
 *   - CUDABackend (include/ternative/ops.h:47-168, cuda/ops_cuda.cu:597-823):
 *     every device method has a tvb_* counterpart below, cited one by one.
 *   - apply_lora (src/model.cpp:205-258) and the INT8 quantizer of
 *     init_gpu_backend (src/model.cpp:374-410), which have no backend hook in
 *     the reference: tvb_merge_i2s_lora / tvb_merge_batch / tvb_quantize_int8.
 *   - Model::forward_gpu (src/model.cpp:1354-1582) and
 *     Model::forward_prefill (src/model.cpp:1139-1234): tvb_decode_step and
 *     tvb_prefill run the same layer order as fused, graph-captured kernels.
 */
#ifndef TVB200_H
#define TVB200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    TVB_OK = 0,
    TVB_ERR_INVALID = 1,      /* bad argument (null pointer, size, alignment) */
    TVB_ERR_CUDA = 2,         /* a CUDA runtime call failed */
    TVB_ERR_OOM = 3,          /* device or pinned allocation failed */
    TVB_ERR_UNSUPPORTED = 4,  /* shape/dtype this build does not handle */
    TVB_ERR_TIMEOUT = 5,      /* a bounded device-side wait gave up */
    TVB_ERR_COMM = 6,         /* tensor-parallel communicator failure */
    TVB_ERR_STATE = 7         /* call out of order (e.g. step before weights set) */
} tvb_status;

/* Weight / output element types. */
typedef enum {
    TVB_F32 = 0,
    TVB_F16 = 1,          /* IEEE half; merge output is the reference's truncating cast */
    TVB_I8_ROW = 2,       /* int8 codes + one F32 scale per output row */
    TVB_I8_TENSOR = 3     /* int8 codes + one F32 scale per tensor (reference INT8) */
} tvb_dtype;

int         tvb_version(void);
const char* tvb_status_string(tvb_status s);
const char* tvb_last_error(void);

/* ------------------------------------------------------------------------ */
/* Device memory helpers — CUDABackend::free_vram_bytes / alloc_gpu_mem /   */
/* upload / release_gpu_mem (ops.h:82-92, ops_cuda.cu:673-692).             */
/* ------------------------------------------------------------------------ */
tvb_status tvb_free_vram_bytes(size_t* free_bytes);
tvb_status tvb_alloc(size_t bytes, void** dptr);
tvb_status tvb_upload(void* dst, const void* src, size_t bytes);   /* synchronous */
/* upload_pinned / download_pinned (ops.h:120-121): synchronous copies. */
tvb_status tvb_download(void* dst_host, const void* src_dev, size_t bytes);
tvb_status tvb_release(void* dptr);

/* ------------------------------------------------------------------------ */
/* Part 1: load-time merge (replaces apply_lora, model.cpp:205-258, and the  */
/* INT8 pass of init_gpu_backend, model.cpp:374-410).                       */
/*                                                                          */
/* One projection W of GGUF ne = [K, N] (stored [N][K], out-major):          */
/*   i2s   : K*N/4 bytes of I2_S codes (K % 128 == 0), the per-tensor scale  */
/*           passed separately (it trails the codes in GGUF, model.cpp:157)  */
/*   A     : lora_a, ne = [K, r], stored [r][K], F32                         */
/*   B     : lora_b, ne = [r, N], stored [N][r], F32                         */
/*   W'    = scale*map(code) + (B.A)*(alpha/r), summed over r in order with  */
/*           unfused F32 multiply/add, exactly as matmul_lora (:192-201)     */
/*   out   : TVB_F32 (merged F32), TVB_F16 (truncating cast, tensor.cpp:33), */
/*           TVB_I8_ROW (per-row absmax/127 of the F16 values, round half    */
/*           away from zero, clip +-127; row_scales gets N floats)           */
/* A == NULL or r == 0 merges nothing (plain unpack + cast).                 */
/* dst must be 16-byte aligned.                                              */
/* ------------------------------------------------------------------------ */
tvb_status tvb_merge_i2s_lora(const uint8_t* i2s, float scale, int K, int N,
                              const float* A, const float* B, int r, float alpha,
                              tvb_dtype out, void* dst, float* row_scales, void* stream);

typedef struct {
    const uint8_t* i2s;
    float scale;
    int K, N;
    const float* A;
    const float* B;
    int r;
    float alpha;
    void* dst;
    float* row_scales;   /* TVB_I8_ROW only */
    /* Column slice, for the tensor-parallel shard of a row-parallel projection
     * (o_proj, down): merge columns [k0, k0 + K) of a tensor whose rows hold
     * ld columns; i2s and A point at the WHOLE tensor's codes and LoRA A
     * ([r][ld]).  Zero (the default) means k0 = 0, ld = K.  k0 and ld are
     * multiples of 128.  A row slice needs no field: offset i2s by
     * row0 * ld / 4 bytes and B by row0 * r floats.  TVB_I8_ROW scales of a
     * column slice come from the slice's own absmax. */
    int k0;
    int ld;
} tvb_merge_desc;

/* All descriptors in one launch (descs is a HOST array of n entries; the
 * device addresses inside it are read on the device).  This is the
 * sharded-by-tensor load-time merge: give each rank its own subset. */
tvb_status tvb_merge_batch(const tvb_merge_desc* descs, int n, tvb_dtype out, void* stream);

/* The same merge with the rank-r delta as a tensor-core contraction
 * (tcgen05.mma on F16 hi + lo splits of A and B, F32 accumulation): TVB_F16
 * output within one unit in the last place of tvb_merge_batch's (which is
 * bit-identical to apply_lora), for ranks up to 64.  TVB_I8_ROW: these F16
 * rows quantised per row exactly as the reference quantises F16 weights
 * (codes within one of tvb_merge_batch's, scales within one F16 unit of the
 * row maximum), through an F16 workspace of at most 512 MB per group of
 * tensors.  F32 output and larger ranks take the tvb_merge_batch path.  Uses
 * a stream-ordered workspace of about 260 B x (N + K) per tensor for the
 * duration of the call. */
tvb_status tvb_merge_batch_tc(const tvb_merge_desc* descs, int n, tvb_dtype out, void* stream);

/* tensor.cpp:1006-1050: I2_S codes -> F32 (n % 128 == 0). */
tvb_status tvb_i2s_unpack(const uint8_t* i2s, int64_t n, float scale, float* out, void* stream);

/* F16 [N][K] -> int8 codes.  per_row != 0: TVB_I8_ROW (scales gets N floats);
 * per_row == 0: the reference's per-tensor quantizer (model.cpp:381-401,
 * scales gets 1 float).  Needs no workspace beyond `scales`. */
tvb_status tvb_quantize_int8(const uint16_t* w_f16, int N, int K, int per_row,
                             int8_t* q, float* scales, void* stream);

/* ------------------------------------------------------------------------ */
/* Part 2 building blocks: the CUDABackend device-pointer API.              */
/* ------------------------------------------------------------------------ */
/* gemv_d2d (ops.h:112-113, ops_cuda.cu:734-740): y[N] = W_f16[N][K] . x[K] */
tvb_status tvb_gemv_f16(float* y, const float* x, const void* W, int K, int N, void* stream);
/* gemv_d2d_int8 (ops.h:116-117, ops_cuda.cu:741-744): y = scale * W_i8 . x */
tvb_status tvb_gemv_int8(float* y, const float* x, const void* W, float scale, int K, int N,
                         void* stream);
/* Per-row INT8 variant: y[n] = row_scales[n] * (W_i8[n] . x). */
tvb_status tvb_gemv_int8_rows(float* y, const float* x, const void* W, const float* row_scales,
                              int K, int N, void* stream);
/* rms_norm_d (ops.h:107-108, ops_cuda.cu:729-733): out = x / sqrt(mean(x^2)+eps) * w */
tvb_status tvb_rms_norm(float* out, const float* x, const float* w, float eps, int N,
                        void* stream);
/* add_d / mul_d / relu2_d (ops.h:102-104, ops_cuda.cu:714-728) */
tvb_status tvb_add(float* out, const float* a, const float* b, int N, void* stream);
tvb_status tvb_mul(float* out, const float* a, const float* b, int N, void* stream);
tvb_status tvb_relu2(float* out, const float* x, int N, void* stream);
/* rope_inplace_d (ops.h:130-131, ops_cuda.cu:757-763): NeoX halves, in place. */
tvb_status tvb_rope_inplace(float* q, float* k, int pos, float theta, int n_heads,
                            int n_kv_heads, int head_dim, void* stream);
/* kv_write_d (ops.h:135, ops_cuda.cu:765-774) on explicit layer slices
 * (k_cache/v_cache point at row 0 of this layer; row stride Hk floats). */
tvb_status tvb_kv_write(const float* k, const float* v, float* k_cache, float* v_cache, int pos,
                        int Hk, void* stream);
/* attention_d (ops.h:141-142, ops_cuda.cu:776-789): one query row against
 * kv_len cached rows, GQA (kv head = h / (n_heads/n_kv_heads)). */
tvb_status tvb_attention_decode(const float* q, const float* k_cache, const float* v_cache,
                                int kv_len, float* out, int n_heads, int n_kv_heads,
                                int head_dim, float scale, void* stream);

/* Weight descriptor (device pointers stay owned by the caller; Tensor::gpu_ptr
 * is non-owning, tensor.h:39-43). */
typedef struct {
    const void* w;          /* weights [N][K] */
    tvb_dtype dtype;        /* TVB_F16, TVB_I8_ROW or TVB_I8_TENSOR */
    const float* row_scales;/* TVB_I8_ROW */
    float tensor_scale;     /* TVB_I8_TENSOR */
} tvb_weight;

/* CUDABackend::matmul / Impl::gemm (ops_cuda.cu:440-491, 600-631) on device
 * buffers: y[M][N] = x[M][K] . W[N][K]^T with F32 activations. */
tvb_status tvb_matmul(float* y, const float* x, int M, int K, const tvb_weight* w, int N,
                      void* stream);

/* Allocation-free split-KV decode attention.  No counterpart in the
 * reference: for callers that cannot allocate device memory when they call
 * (a host that hands its device memory to its own pool at start-up, or a
 * thread that must not risk the device synchronisation cudaMalloc/cudaFree
 * can imply).  Same arguments and result as tvb_attention_decode; its split
 * partials live in a static device array inside this library (64 heads x 8
 * splits x head_dim 128, 264 KiB, held by every GPU that loads the library
 * until the process exits).  n_heads > 64 is rejected with TVB_ERR_INVALID.
 * The first call on a device looks up that array's device address (make it
 * with the device current, before any stream capture).  Every call shares the
 * array: calls that overlap on the GPU (other streams, other threads) race. */
tvb_status tvb_attention_decode_noalloc(const float* q, const float* k_cache, const float* v_cache,
                                        int kv_len, float* out, int n_heads, int n_kv_heads,
                                        int head_dim, float scale, void* stream);

/* ------------------------------------------------------------------------ */
/* Context: the state CUDABackend::Impl owns (ops_cuda.cu:309-591):         */
/* stream, activation buffers, KV cache, pinned staging, workspace, plus    */
/* the fused decode/prefill step over a registered weight table.            */
/* ------------------------------------------------------------------------ */
typedef struct {
    int vocab_size;
    int hidden_size;
    int num_layers;
    int num_heads;
    int num_kv_heads;
    int head_dim;
    int intermediate_size;
    int max_seq_len;     /* device KV capacity (the reference hard-codes 1024) */
    float rope_theta;
    float rms_norm_eps;
    int max_prefill;     /* largest prefill batch (0 -> 1024) */
    int max_batch;       /* KV cache slots for batched decode (0 -> 1) */
} tvb_model_config;

typedef struct tvb_context tvb_context;

/* init_gpu_activations (ops.h:93, ops_cuda.cu:355-395).  Allocates on the
 * current device; creates its own non-blocking stream. */
tvb_status tvb_context_create(const tvb_model_config* cfg, tvb_context** out);
tvb_status tvb_context_destroy(tvb_context* ctx);
void*      tvb_context_stream(tvb_context* ctx);

/* d_x()/d_norm()/d_q()/d_k()/d_v()/d_gate()/d_up() and h_qkv()/h_attn()/
 * h_logit() (ops.h:94-110). */
typedef struct {
    float* d_x;
    float* d_norm;
    float* d_q;
    float* d_k;
    float* d_v;
    float* d_gate;
    float* d_up;
    float* h_qkv;
    float* h_attn;
    float* h_logit;
} tvb_buffers;
tvb_status tvb_context_buffers(tvb_context* ctx, tvb_buffers* out);

/* clear_kv_d / has_gpu_kv / gpu_kv_max_seq / upload_kv_layer_d /
 * download_kv_slot_d (ops.h:145-162).  KV layout: [layer][pos][Hk] F32. */
tvb_status tvb_kv_clear(tvb_context* ctx);
int        tvb_kv_capacity(tvb_context* ctx);
tvb_status tvb_kv_layer_ptrs(tvb_context* ctx, int layer, float** k, float** v);
tvb_status tvb_kv_upload_layer(tvb_context* ctx, int layer, int n_positions, const float* h_k,
                               const float* h_v);
tvb_status tvb_kv_download_slot(tvb_context* ctx, int layer, int pos, int n_floats, float* h_dst);
/* sync_d (ops.h:123). */
tvb_status tvb_context_sync(tvb_context* ctx);

/* Phase trace of the fused decode step (no counterpart in the reference, whose
 * only tracing is stdout progress lines).  Only the trace build of the library
 * (libtvb200_trace.so, `make -C ternative_b200/csrc trace`) records: every
 * later decode-step launch on this device writes, from thread 0 of each CTA,
 * %globaltimer nanoseconds at 8 event slots per (phase, CTA) into `dev_buf`
 * laid out [phase][CTA][8] as 64-bit words, for the first `n_phases` phases
 * (the buffer holds n_phases x SMs x 8 words).  Slots: 0 phase start, 1 inputs
 * staged, 2 weight stream done, 3 epilogue done, 6 barrier arrival, 4 next
 * phase prepared, 5 barrier passed.  dev_buf NULL stops tracing.
 * The product build returns TVB_ERR_UNSUPPORTED. */
tvb_status tvb_trace_set(void* dev_buf, int n_phases);

/* ------------------------------------------------------------------------ */
/* Tensor parallelism: one process (and context) per GPU.  No counterpart in */
/* the reference, whose GPU path is single-device.  Each rank's context is  */
/* created with its shard's dimensions (num_heads, num_kv_heads and          */
/* intermediate_size divided by the ranks; hidden_size and vocab_size whole) */
/* and registered with its shard of every projection: q/k/v and gate/up are */
/* split by rows, o_proj and down by columns (tvb_merge_desc k0/ld), the    */
/* tied lm_head by vocabulary rows (tvb_set_output still takes the whole    */
/* embedding table).  The decode step then exchanges partial rows with the  */
/* other ranks over NVLink inside its single launch, after o_proj and after */
/* down, and agrees on the argmax across vocabulary slices.                  */
/*                                                                          */
/* Setup: tvb_tp_init on every rank returns this rank's exchange buffer;    */
/* export it with tvb_ipc_export, give the handles to every rank, import    */
/* the others' with tvb_ipc_import and pass all buffers (own at [rank]) to  */
/* tvb_tp_set_peers.  Every rank must then run the same sequence of decode  */
/* and prefill calls; logits returned are this rank's vocabulary slice       */
/* (vocab_size / world floats, rows [rank * vocab_size / world, ...)).      */
/* When a step's device-side wait gives up (TVB_ERR_TIMEOUT, e.g. a rank    */
/* skipped the step), the ranks' exchange counters no longer agree: that    */
/* rank then refuses steps (TVB_ERR_STATE) until tvb_tp_recover.  Recover   */
/* every rank (each call zeroes that rank's exchange buffer and step        */
/* counters after its stream is idle), and let no rank start a step before  */
/* all ranks have returned from tvb_tp_recover (a host-side barrier).       */
/* Close imported buffers (tvb_ipc_close) after destroying the context.     */
/* ------------------------------------------------------------------------ */
typedef struct {
    unsigned char bytes[64];
} tvb_ipc_handle;

tvb_status tvb_tp_init(tvb_context* ctx, int rank, int world, void** exchange);
tvb_status tvb_tp_set_peers(tvb_context* ctx, void* const* exchanges);
tvb_status tvb_tp_recover(tvb_context* ctx);
tvb_status tvb_ipc_export(const void* dev_ptr, tvb_ipc_handle* out);
tvb_status tvb_ipc_import(const tvb_ipc_handle* handle, void** dev_ptr);
tvb_status tvb_ipc_close(void* dev_ptr);

/* Weight table for the fused step. */
typedef struct {
    const float* attn_norm;     /* [H]  */
    tvb_weight wq, wk, wv;      /* [Hq][H], [Hk][H], [Hk][H] */
    const float* attn_sub_norm; /* [Hq] */
    tvb_weight wo;              /* [H][Hq] */
    const float* ffn_norm;      /* [H]  */
    tvb_weight w_gate, w_up;    /* [I][H] */
    const float* ffn_sub_norm;  /* [I]  */
    tvb_weight w_down;          /* [H][I] */
} tvb_layer_weights;

tvb_status tvb_set_layer(tvb_context* ctx, int layer, const tvb_layer_weights* lw);
/* tok_embd F16 [V][H] (tied lm_head, model.cpp:1579) and output_norm F32 [H]. */
tvb_status tvb_set_output(tvb_context* ctx, const void* tok_embd_f16, const float* output_norm);

/* Model::forward_gpu (model.cpp:1354-1582) for one token at position `pos`
 * (KV rows [0, pos) must be filled): embedding, all layers, final norm and
 * the lm_head on the device.  logits_host (V floats, may be NULL) and
 * argmax_host (may be NULL) are filled from pinned staging; this call
 * synchronises its stream. */
tvb_status tvb_decode_step(tvb_context* ctx, int token, int pos, float* logits_host,
                           int* argmax_host);

/* Greedy decode of n_steps tokens entirely on the device: step i feeds the
 * argmax of step i-1 back as its token.  Starts from `token` at `pos`.
 * tokens_host receives n_steps argmax ids.  Synchronises. */
tvb_status tvb_generate_greedy(tvb_context* ctx, int token, int pos, int n_steps,
                               int* tokens_host);

/* Enqueue n_steps chained greedy steps (as tvb_generate_greedy) on the
 * context stream and return without synchronising; argmax ids accumulate in
 * device memory.  For timing and for overlapping host work. */
tvb_status tvb_decode_enqueue(tvb_context* ctx, int token, int pos, int n_steps);

/* Model::forward_prefill (model.cpp:1139-1234) over S tokens starting at
 * position 0: fills KV rows [0, S) and returns the logits of the last row
 * (and its argmax).  Synchronises. */
tvb_status tvb_prefill(tvb_context* ctx, const int* tokens_host, int S, float* last_logits_host,
                       int* argmax_host);

/* Batched decode of up to max_batch independent sequences (no reference
 * counterpart: the reference serves one sequence; its batch of 8 is 8
 * sequential Model::forward_gpu runs, model.cpp:1354-1582).  Sequence b lives
 * in KV cache slot b.
 *
 * tvb_prefill_slot: tvb_prefill into slot `slot` (slot 0 is the KV cache of
 * the single-sequence calls); like tvb_prefill it leaves the step state at
 * (S, argmax).
 *
 * tvb_decode_batch: one greedy step of sequences 0 .. B-1: tokens[b] at
 * positions[b] of slot b (KV row positions[b] is written, attention over rows
 * [0, positions[b]]).  next_tokens[b] = argmax of row b's logits; logits
 * (optional, host [B][vocab / tp_world], this rank's slice) receives them.
 * Every weight byte is read once for all B rows (tensor-core GEMM with B
 * activation rows).  Synchronises. */
tvb_status tvb_prefill_slot(tvb_context* ctx, int slot, const int* tokens_host, int S,
                            float* last_logits_host, int* argmax_host);
tvb_status tvb_decode_batch(tvb_context* ctx, const int* tokens_host, const int* positions_host, int B,
                            float* logits_host, int* next_tokens_host);

/* Model::score_logprobs (model.cpp:1746-1831): prefill the T tokens (KV slot 0)
 * and, for every position p in [max(1, start_pos), T), the log-probability of
 * tokens[p] given tokens[0, p) (logprobs[p - first]) and the k largest
 * log-probabilities with their ids (top_*[(p - first) * k + j], descending).
 * k <= 64; single-GPU contexts.  Synchronises. */
tvb_status tvb_score_logprobs(tvb_context* ctx, const int* tokens_host, int T, int start_pos, int k,
                              float* logprobs_host, int* top_ids_host, float* top_logprobs_host);

/* ---- token sampler --------------------------------------------------------
 * sample_token (src/sampler.cpp:11-148; SamplerConfig, include/ternative/
 * sampler.h:8-14) on the device for B rows of logits (row b at logits + b*ld):
 * temperature, repetition penalty over row b's seen tokens (seen + b*max_seen,
 * n_seen[b] of them), softmax, top-k, top-p, renormalisation and the draw
 * against u[b] in [0, 1) (the reference draws it from its own mt19937).
 * out[b] receives the token.  All pointers are device memory.  top_p in (0, 1)
 * with top_k 0 (the whole vocabulary) or above 1024 takes a one-CTA-per-row
 * kernel that walks the sorted probabilities 1024 at a time (slower for flat
 * distributions, whose nucleus holds many tokens).  Allocates a per-call
 * workspace on `stream`. */
typedef struct {
    float temperature;
    float top_p;
    int top_k;
    float repetition_penalty;
} tvb_sampler_config;

tvb_status tvb_sample(const float* logits, int B, int vocab, int ld, const tvb_sampler_config* cfg,
                      const int* seen, const int* n_seen, int max_seen, const float* u, int* out, void* stream);

/* ---- merged-weight cache (.tvcache) ---------------------------------------
 * ModelCache::save / ModelCache::try_load (src/cache.cpp:263-470, format
 * include/ternative/cache.h:28-62), fed from and into device memory: the merge
 * output is written without a host copy of the model, and a cached model is
 * uploaded chunk by chunk.  Files without INT8 tensors are byte-identical to
 * the reference's (version 1); per-row INT8 weights (ggml type 24 plus an F32
 * "<name>.row_scale" entry) make a version-2 file, which the reference's
 * reader refuses.  Pointers may be host or device memory. */
typedef struct {
    uint64_t base_size;        /* the reference writes 0 */
    uint8_t base_sha256[32];   /* SHA-256 of the base GGUF (ModelCache::compute_key) */
    uint64_t lora_size;        /* the reference writes 0 */
    uint8_t lora_sha256[32];   /* zeros without LoRA */
    float lora_alpha;
    uint32_t lora_rank;
} tvb_cache_key;

typedef struct {
    const char* name;          /* "tok_embd", "output_norm", "blk.<l>.attn_q", ... */
    int ggml_type;             /* 0 F32, 1 F16, 24 I8 (per-row INT8 codes) */
    int n_dims;                /* 1..4 */
    int64_t shape[4];          /* ggml order: shape[0] = ne0 (the row length) */
    const void* data;
    const float* row_scales;   /* I8: shape[1] F32 scales */
} tvb_cache_tensor;

typedef struct tvb_cache tvb_cache;

/* Writes `path` (via <path>.tmp and a rename, as ModelCache::save). */
tvb_status tvb_cache_write(const char* path, const tvb_cache_key* key, const tvb_cache_tensor* tensors, int n);
/* Opens a cache file and reads its header and tensor table. */
tvb_status tvb_cache_open(const char* path, tvb_cache** out);
int        tvb_cache_count(const tvb_cache* cache);
tvb_status tvb_cache_info(const tvb_cache* cache, tvb_cache_key* key, int* version);
/* Entry i: name (valid while open), type, dims, shape; data pointers unset. */
tvb_status tvb_cache_entry(const tvb_cache* cache, int i, tvb_cache_tensor* info, uint64_t* nbytes);
/* Reads tensor `name` into dst (capacity bytes, host or device). */
tvb_status tvb_cache_read(tvb_cache* cache, const char* name, void* dst, uint64_t capacity);
tvb_status tvb_cache_close(tvb_cache* cache);

/* ---- GGUF ingest -----------------------------------------------------------
 * gguf_load (src/gguf.cpp:220-249, parse :254-307) reads the whole file into
 * host memory.  These read only the header and tensor table, then stream one
 * tensor at a time from the file into device (or host) memory through pinned
 * staging -- e.g. the I2_S codes and LoRA factors straight into the merge's
 * inputs.  Sizes as the reference's Tensor (tensor.cpp:108-121): F32, F16,
 * BF16 and I2_S (32 bytes per 128 weights + the F32 scale). */
typedef struct tvb_gguf tvb_gguf;
tvb_status tvb_gguf_open(const char* path, tvb_gguf** out);
int        tvb_gguf_count(const tvb_gguf* gguf);
/* Entry i: name (valid while open), ggml type, dims, shape; nbytes 0 for types
 * this reader does not size. */
tvb_status tvb_gguf_tensor(const tvb_gguf* gguf, int i, tvb_cache_tensor* info, uint64_t* nbytes);
tvb_status tvb_gguf_read(tvb_gguf* gguf, const char* name, void* dst, uint64_t capacity);
tvb_status tvb_gguf_close(tvb_gguf* gguf);

#ifdef __cplusplus
}
#endif
#endif /* TVB200_H */
