/*
 * cuda_inference.h — C ABI of the B200 (sm_100a) batch-1 Qwen3 decode engine.
 *
 * It is the surface of the reference's GPU engine, metal_infrence_engine/src/metal_inference.rs,
 * re-expressed as plain C so that a thin `cuda_inference.rs` (or ctypes/cffi) can bind it and drop
 * it in beside the reference CPU engine, metal_infrence_engine/src/cpu_inference.rs. Each
 * declaration names the reference item it replaces (path:line inside metal_infrence_engine/).
 *
 * Conventions (where the reference panics, these return a status code):
 *   - every int-returning call returns QW_OK (0) or a QW_ERR_* code; qw_last_error() gives the
 *     message of the calling thread's most recent failure;
 *   - the caller owns handles and frees them with the matching *_free;
 *   - a model is bound to one CUDA device and owns one stream; calls on one handle are not
 *     thread-safe; different handles (one per device) may be driven from different threads;
 *   - host pointers are plain host memory; `d_` pointers are device memory on the model's device;
 *     `stream` is a cudaStream_t (NULL = the model's own stream).
 */
#ifndef CUDA_INFERENCE_H
#define CUDA_INFERENCE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    QW_OK = 0,
    QW_ERR_IO = 1,             /* file missing / unreadable (reference: io::Error from load_model) */
    QW_ERR_FORMAT = 2,         /* malformed safetensors/config, missing tensor, wrong shape */
    QW_ERR_UNSUPPORTED = 3,    /* non-BF16 tensor, geometry the kernels do not support */
    QW_ERR_ARG = 4,            /* bad argument: token >= vocab, pos >= max_seq, NULL handle */
    QW_ERR_CUDA = 5,           /* CUDA runtime error (no device, launch failure, ...) */
    QW_ERR_DEVICE_TIMEOUT = 6, /* a bounded device-side wait expired; the kernel stopped cleanly */
    QW_ERR_NOMEM = 7           /* device or pinned host allocation failed */
};

typedef struct qw_model qw_model;
typedef struct qw_cache qw_cache;

/* cpu_inference.rs:21-33 Config (the ten config.json fields the reference reads) */
typedef struct qw_config {
    uint64_t hidden_size;
    uint64_t intermediate_size;
    uint64_t num_hidden_layers;
    uint64_t num_attention_heads;
    uint64_t num_key_value_heads;
    uint64_t head_dim;
    uint64_t vocab_size;
    float rms_norm_eps;
    float rope_theta;
    uint32_t eos_token_id;
} qw_config;

/* message of this thread's most recent failure ("" if none) */
const char* qw_last_error(void);

/* Parse and validate `safetensors_path` and the config.json beside it without touching a GPU.
 * Replaces the parsing half of Model::load_model (cpu_inference.rs:58-84). */
int qw_inspect(const char* safetensors_path, qw_config* out);

/* MetalModel::load_model (metal_inference.rs:157-168): parse, validate, upload (repacked) to
 * `device`. */
int qw_load(const char* safetensors_path, int device, qw_model** out);
void qw_free(qw_model* model);

/* MetalModel::config (metal_inference.rs:170) */
int qw_config_get(const qw_model* model, qw_config* out);

/* bytes one decode token reads by the reference's rule (tests/mbu.rs:19-30, bench.rs:107-116):
 * every tensor except the embedding table, plus one bf16 embedding row */
uint64_t qw_weight_bytes_per_token(const qw_model* model);

/* MetalKVCache::new (metal_inference.rs:129-137): f32 K/V for `max_seq` positions and the RoPE
 * table. Unlike the reference (max_seq <= 4064, metal_inference.rs:130) the only cap is memory. */
int qw_cache_new(qw_model* model, size_t max_seq, qw_cache** out);
void qw_cache_free(qw_cache* cache);
size_t qw_cache_max_seq(const qw_cache* cache); /* MetalKVCache::max_seq (metal_inference.rs:121) */

/* MetalModel::forward (metal_inference.rs:286-291): run `token` at `pos`, write its K/V into the
 * cache, copy vocab_size f32 logits to `logits_out` (host). Synchronous. */
int qw_forward(qw_model* model, qw_cache* cache, uint32_t token, size_t pos, float* logits_out);

/* Batched prefill (the 512-token prompt workload; the reference feeds a prompt token by token through
 * forward, metal_inference.rs:286-291, src/bin/bench.rs:166-191): one pass over ids[0..n) at
 * positions start_pos .. start_pos+n-1 whose projections run as tcgen05 tensor-core GEMMs over all
 * n tokens. Writes their K/V into the cache exactly where n forward calls would; with logits_out
 * (host, n * vocab_size floats, row t = position start_pos + t) also every position's logits.
 * Synchronous. logits_out must be host memory (a device pointer is refused with QW_ERR_ARG before
 * any work). A page-locked logits_out (cudaHostAlloc, cudaHostRegister, a pinned torch tensor) is
 * filled by one DMA; pageable memory of 32 MB or more goes through two 16 MB pinned stages that the
 * model allocates on first use and up to 8 host threads copy out (311 MB for 512 positions: 8.6 ms
 * page-locked, 9.9 ms into pageable memory written before, 18 ms into a new array). */
int qw_prefill(qw_model* model, qw_cache* cache, const uint32_t* ids, size_t n, size_t start_pos, float* logits_out);
/* qw_prefill with device-resident ids (d_ids[n]) and logits (d_logits[n * vocab_size] or NULL),
 * stream-ordered on `stream` (NULL = the model's stream), without synchronisation; token ids are not
 * range-checked here (they must be < vocab_size). A GEMM wait that expired is reported by qw_sync. */
int qw_prefill_device(qw_model* model, qw_cache* cache, const uint32_t* d_ids, size_t n, size_t start_pos,
                      float* d_logits, void* stream);

/* Batch decode (the box workload's per-GPU batch-8 variant): B independent sequences, each
 * with its own cache, advance one token per step together, so each step streams the weights once
 * for all B (the reference decodes one sequence per engine, metal_inference.rs:286-387). Every
 * projection is a tcgen05 GEMM over the B rows; attention runs per row over the row's own cache.
 * 1 <= B <= QW_BATCH_MAX; the caches must be distinct and belong to `model`.
 *
 * qw_forward_batch: row b feeds tokens[b] at positions[b] into caches[b] (forward() for each row,
 * metal_inference.rs:286); logits_out is B * vocab_size floats, row b at b * vocab_size. Synchronous.
 *
 * qw_decode_batch: decode() for each row (metal_inference.rs:297): firsts[b] goes in at
 * start_pos[b], each step's argmax feeds the row's next step, and tokens_out[b * steps + i] receives
 * row b's i-th output token. One step is captured once as a CUDA graph and replayed. Synchronous.
 *
 * qw_decode_batch_device: the same with device first tokens (d_firsts[B]) and a device token
 * record d_out[steps * B] in step-major order (d_out[i * B + b]), stream-ordered on `stream`
 * (NULL = the model's stream) without synchronisation; start_pos stays a host array. */
#define QW_BATCH_MAX 16
int qw_forward_batch(qw_model* model, qw_cache* const* caches, size_t B, const uint32_t* tokens, const size_t* positions,
                     float* logits_out);
int qw_decode_batch(qw_model* model, qw_cache* const* caches, size_t B, const uint32_t* firsts, const size_t* start_pos,
                    size_t steps, uint32_t* tokens_out);
int qw_decode_batch_device(qw_model* model, qw_cache* const* caches, size_t B, const uint32_t* d_firsts,
                           const size_t* start_pos, size_t steps, uint32_t* d_out, void* stream);

/* Prompt-lookup speculative greedy decode (the reference's proposed route past one token per weight
 * pass, README.md:109-111: "same greedy output with more than one token per pass"). Same contract
 * as qw_decode (`first` goes in at start_pos, `steps` greedy output tokens into tokens_out), plus
 * the token history `context[0..context_len)` (e.g. the prompt) that drafts are looked up in. Per
 * pass: the longest n-gram of at most max_ngram tokens that ends the history (context, first and
 * the tokens produced so far) and occurred earlier proposes the draft_max tokens that followed its
 * latest earlier occurrence (continued periodically where that occurrence overlaps the end of the
 * history); one multi-token forward over the current token and the draft (tcgen05 GEMMs, as
 * qw_prefill, captured as a graph) checks them all, and the matching prefix plus the next greedy
 * token are emitted. Without a draft of at least 2 tokens a pass is one decode-kernel step.
 * Positions written for rejected drafts are overwritten by later passes. stats (may be NULL)
 * counts passes, drafted and accepted tokens. Synchronous. */
#define QW_LOOKUP_DRAFT_MAX 15
typedef struct {
    uint64_t passes;    /* forward passes (verify passes and single decode steps) */
    uint64_t drafted;   /* draft tokens proposed */
    uint64_t accepted;  /* draft tokens accepted */
} qw_lookup_stats;
int qw_decode_lookup(qw_model* model, qw_cache* cache, const uint32_t* context, size_t context_len, uint32_t first,
                     size_t start_pos, size_t steps, uint32_t max_ngram, uint32_t draft_max, uint32_t* tokens_out,
                     qw_lookup_stats* stats);

/* MetalModel::decode (metal_inference.rs:297-316): greedy decode; `first` goes in at `start_pos`,
 * each step's argmax feeds the next, and on_token(user, t) is called with each step's output
 * token as soon as the GPU produces it (steps calls). The whole run is one kernel launch. */
typedef void (*qw_token_fn)(void* user, uint32_t token);
int qw_decode(qw_model* model, qw_cache* cache, uint32_t first, size_t start_pos, size_t steps,
              qw_token_fn on_token, void* user);

/* Device-resident variants of forward/decode (no host copies, no synchronisation): stream-ordered
 * launches for callers that keep tokens and logits on the GPU (benchmarks, servers).
 * d_tokens has steps + 1 entries: d_tokens[0] is the input, d_tokens[i + 1] receives step i's
 * argmax (the ring of metal_inference.rs:298-302). Errors raised on the device are reported by
 * the next qw_sync. */
int qw_forward_device(qw_model* model, qw_cache* cache, const uint32_t* d_token, size_t pos,
                      float* d_logits, void* stream);
int qw_decode_device(qw_model* model, qw_cache* cache, uint32_t* d_tokens, size_t start_pos,
                     size_t steps, void* stream);
int qw_sync(qw_model* model, void* stream);

/* Copy layer `layer`'s K and V for positions [0, n) to host buffers in the reference layout
 * [t][num_key_value_heads * head_dim] (KVCache, cpu_inference.rs:44-48). */
int qw_cache_read(qw_cache* cache, size_t layer, size_t n, float* k_out, float* v_out);

/* Streaming-SM count the decode kernel uses (one CTA per SM). */
int qw_num_ctas(const qw_model* model);

/* Which decode kernel runs qw_forward / qw_decode for this model (no reference counterpart: the
 * reference has one Metal pipeline per op). QW_DECODER_GRID, the default: one CTA per SM over the
 * whole GPU, every shape. QW_DECODER_CLUSTER, when the environment sets QW_DECODER=cluster at
 * load: 8 thread-block clusters of 8 CTAs, one per KV head, exchanging activations through
 * distributed shared memory (the Qwen3-0.6B layer shape only). Both compute the same function
 * (cpu_inference.rs:100-179). */
#define QW_DECODER_GRID 0
#define QW_DECODER_CLUSTER 1
int qw_decoder_kind(const qw_model* model);

/* How qw_decode_batch runs batches of at most 8 rows (no reference counterpart: the reference
 * decodes one sequence per engine, metal_inference.rs:286-387). QW_BATCH_ROWS, the default: a
 * captured graph of row-mode kernels per step (skinny tensor-core GEMMs, row attention).
 * QW_BATCH_PERSISTENT, when the environment sets QW_BATCH_DECODER=persistent at load and the
 * model's shapes fit: one persistent launch for all steps, streaming the weights once per step
 * for every row (batch_kernel.cuh). Batches of 9 to 16 rows always run in row mode. -1 for a null
 * model. */
#define QW_BATCH_ROWS 0
#define QW_BATCH_PERSISTENT 1
int qw_batch_decoder_kind(qw_model* model);

/* The model's own cudaStream_t (what qw_forward/qw_decode run on), e.g. to bracket them with
 * events. */
void* qw_model_stream(const qw_model* model);

/* Phase timeline (tracing): when enabled, every launch records, for its first step, per CTA,
 * qw_trace_stride() globaltimer stamps (ns): 14 per layer at the phase hand-offs, then 4 for the
 * lm_head / argmax tail. qw_read_trace copies num_ctas * stride stamps of the most recent launch.
 * The reference measured its per-part breakdown by ablation (README.md:64-71); this records it. */
size_t qw_trace_stride(const qw_model* model);
int qw_set_trace(qw_model* model, int enable);
int qw_read_trace(qw_model* model, uint64_t* out, size_t capacity);

/* ---- standalone kernels (the device code of the decode kernel, exposed for microbenchmarks) ---- */

/* y = W x, W bf16 [rows][cols] row-major, x/y f32 — the matvec_bf16 kernel
 * (src/shaders/inference.metal:143-186, cpu_inference.rs:225-257) as the decode kernel streams it.
 * cols must split into 1, 2, 3, 4, 6 or 12 segments of 256, 512, 768 or 1024 columns
 * (e.g. 256, 512, 768, 1024, 2048, 3072, 4096, 6144, 12288). */
int qw_gemv_bf16(int device, const uint16_t* d_w, const float* d_x, float* d_y, size_t rows, size_t cols,
                 void* stream);

/* The same GEMV over `count` matrices of one shape stored back to back (d_w [count][rows][cols],
 * d_y [count][rows], one x) in ONE launch: every CTA owns the same rows of each matrix as in
 * qw_gemv_bf16 and streams matrix after matrix, the way the decode kernel streams layer after layer.
 * It measures the steady-state streaming rate of a layer-sized shape, which a single launch of a
 * few MB cannot show (the reference's tests/read_bandwidth.rs:69-141 likewise
 * times many passes back to back). count >= 1. */
int qw_gemv_bf16_seq(int device, const uint16_t* d_w, const float* d_x, float* d_y, size_t rows, size_t cols,
                     size_t count, void* stream);

/* *d_out = first index of the largest element (tests/common/mod.rs:17-22: ties to the lowest
 * index, a NaN at index 0 gives 0, other NaNs never win; the GPU argmax of
 * shaders/inference.metal:300-321). d_workspace holds qw_argmax_workspace_size(n) bytes. */
size_t qw_argmax_workspace_size(size_t n);
int qw_argmax_f32(int device, const float* d_x, size_t n, uint32_t* d_out, void* d_workspace, void* stream);

/* qw_argmax_f32 for callers that cannot allocate device memory — for example code running inside
 * a CUDA stream capture, or a host that owns the device allocator and forbids cudaMalloc on its
 * serving path. This entry point has no counterpart in the reference. Instead of a caller
 * workspace it uses one file-scope device array of 8,448 bytes that every GPU loading this
 * library holds until the process exits; it calls no cudaMalloc, cudaFree or other allocating
 * routine. The first call on a device looks up that array's device address (do it before any
 * stream capture). n must be in [1, QW_ARGMAX_NOALLOC_MAX_N]; larger n returns QW_ERR_ARG. All
 * calls on a device share the array, which keeps the last call's contents (the call clears what
 * must start at zero itself): two calls that overlap on the GPU — on different streams, or from
 * different threads — race and give wrong results; keep them ordered on one stream. The looked-up
 * address is kept for the life of the process: a cudaDeviceReset on that device invalidates it
 * (and every handle of this library on the device), so do not reset a device this library uses. */
#define QW_ARGMAX_NOALLOC_MAX_N 4294967295ull
int qw_argmax_f32_noalloc(int device, const float* d_x, size_t n, uint32_t* d_out, void* stream);

/* The batched prefill's tensor-core GEMM (tcgen05, TMA tiles): d_y[M][N] (f32) =
 * (d_a_hi + d_a_lo)[M][K] . d_b[N][K]^T, where d_a_hi / d_a_lo are the bf16 high and low halves of
 * f32 activations and d_b a bf16 weight matrix [out][in] as stored (matvec_bf16's operand,
 * src/shaders/inference.metal:143-186, for many tokens at once). K must be a multiple of 64 and
 * every pointer 16-byte aligned. Synchronous: returns after the product is in d_y. */
int qw_gemm_bf16x2(int device, const uint16_t* d_a_hi, const uint16_t* d_a_lo, const uint16_t* d_b, float* d_y, size_t M,
                   size_t N, size_t K, void* stream);

/* Streaming-read probe (tests/read_bandwidth.rs:16-54): sums n_floats floats (n_floats % 4 == 0,
 * d_src 16-byte aligned) into per-CTA partials d_partials[0 .. n_partials). Returns the number
 * of partials written through *n_written. */
int qw_read_probe(int device, const float* d_src, size_t n_floats, float* d_partials, size_t n_partials,
                  size_t* n_written, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* CUDA_INFERENCE_H */
