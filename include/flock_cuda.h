/*
 * flock_cuda.h -- C ABI of libflock_cuda.so, the B200 (sm_100a) replacement
 * for flock's per-token Qwen3 hot path (the kernels/ module of
 * ethanhinson/flock).  Plain C types only: a Deno.dlopen / ctypes / cgo
 * binding can bind every symbol below without a C++ or CUDA header.
 *
 * Conventions
 *  - Every call returns an int status: FLOCK_OK (0) or a negative FLOCK_E_*
 *    code; flock_last_error() returns the calling thread's message, worded
 *    like the reference's thrown Error where one exists.
 *  - Host pointers passed in are read during the call and not retained;
 *    host output pointers are written before the call returns (the call
 *    synchronises the handle's stream when it returns data to the host).
 *  - Handles are opaque.  A handle is bound to one device and one CUDA
 *    stream and is not thread-safe (the reference is single-threaded: one JS
 *    event loop, one conversation, docs/ARCHITECTURE.md:295-296).
 *  - Matrices are [rows][cols] row-major, rows = output size, cols = input
 *    size (GGUF lists the shape as [cols, rows]; kernels/layer.ts:20-22).
 *
 * Reference interfaces are cited as file:line within ethanhinson/flock.
 */
#ifndef FLOCK_CUDA_H
#define FLOCK_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(FLOCK_BUILD)
#define FLOCK_API __attribute__((visibility("default")))
#else
#define FLOCK_API
#endif

#define FLOCK_OK 0
#define FLOCK_E_ARG (-1)     /* bad argument / shape (reference: throw new Error) */
#define FLOCK_E_CUDA (-2)    /* CUDA runtime error */
#define FLOCK_E_STATE (-3)   /* KV cache full, offset mismatch, maxPrefill exceeded */
#define FLOCK_E_MISSING (-4) /* a required tensor is missing (layer.ts:269-287) */
#define FLOCK_E_LIMIT (-5)   /* a shard does not fit its binding/memory limit (shard.ts:229-243) */
#define FLOCK_E_NCCL (-6)    /* NCCL error or timeout */
#define FLOCK_E_NOMEM (-7)   /* device allocation failed */
#define FLOCK_E_UNSUPPORTED (-8)

#define FLOCK_Q8_0 8  /* 34-byte blocks: f16 scale + 32 int8 (lib.ts:25-26) */
#define FLOCK_Q4_0 4  /* 18-byte blocks: f16 scale + 16 nibble pairs (lib.ts:27-28) */
#define FLOCK_F32 32  /* plain f32 (norm gains) */

#define FLOCK_ROPE_NEOX 0 /* pairs (j, j+hd/2): HuggingFace halves (lib.ts:526) */
#define FLOCK_ROPE_NORM 1 /* pairs (2j, 2j+1): GGUF adjacent */

#define FLOCK_ATTN_EXACT 0 /* decode attention in attnRef's exact order (ops_ref.ts:135) */
#define FLOCK_ATTN_FAST 1  /* split-K flash-decode; no key cap; tolerance 1e-5 rel */

#define FLOCK_PREFILL_EXACT 0  /* prefill in the reference's f32 order (bit-exact) */
#define FLOCK_PREFILL_TENSOR 1 /* prefill matmuls and attention on the tcgen05 tensor cores:
                                  16-bit (f16) operands, f32 accumulation, max relative
                                  error 1e-2 */

#define FLOCK_KV_F32 0  /* f32 KV cache, the reference's (layer.ts:394-397 kcache/vcache) */
#define FLOCK_KV_BF16 1 /* bf16 KV cache: half the bytes per key; each appended key and
                           value is rounded to nearest even once and every attention
                           read widens it exactly.  Needs FLOCK_ATTN_FAST and
                           FLOCK_PREFILL_TENSOR (the exact kernels are f32 only). */
#define FLOCK_KV_FP8 2  /* fp8 KV cache (OCP E4M3FN): a quarter of the bytes per key;
                           each appended key and value is rounded to the nearest e4m3
                           (ties to even, magnitudes past 448 saturate to 448, no
                           scale) once and every read widens it exactly.  Needs
                           FLOCK_ATTN_FAST and FLOCK_PREFILL_TENSOR. */

#define FLOCK_MATVEC_EXACT 0 /* one-token matvecs in cpuMatmulQ8F32(coop(64))'s f32 order
                                (lib.ts:213), bit-identical */
#define FLOCK_MATVEC_FAST 1  /* the decode LM head (output_norm + matvec + argmax) on the int8
                                tensor cores: x split into three int8 digits per 32-block,
                                exact int32 block sums, f32 scaling; reassociated, max
                                relative error 1e-3 (measured ~1e-6) */

typedef struct flock_dev flock_dev;
typedef struct flock_tensor flock_tensor;
typedef struct flock_layer flock_layer;
typedef struct flock_model flock_model;
typedef struct flock_shard flock_shard;
typedef struct flock_head flock_head;
typedef struct flock_comm flock_comm;

/* kernels/layer.ts:87-112 LayerConfig (+ the decode-attention choice). */
typedef struct flock_layer_config {
  int32_t hidden;       /* 1024 */
  int32_t n_heads;      /* 16 */
  int32_t n_kv_heads;   /* 8 */
  int32_t head_dim;     /* 128 (the kernels require 128) */
  int32_t ffn;          /* 3072 */
  float eps;            /* f32(1e-6) */
  double rope_base;     /* 1e6 */
  int32_t max_keys;     /* KV cache capacity */
  int32_t max_prefill;  /* largest prefill batch (sizes activations) */
  int32_t rope_pairing; /* FLOCK_ROPE_NEOX | FLOCK_ROPE_NORM */
  int32_t attention;    /* FLOCK_ATTN_EXACT | FLOCK_ATTN_FAST */
  int32_t prefill;      /* FLOCK_PREFILL_EXACT | FLOCK_PREFILL_TENSOR (multi-token steps) */
  int32_t kv_dtype;     /* FLOCK_KV_F32 (0, the default) | FLOCK_KV_BF16 | FLOCK_KV_FP8 */
  int32_t matvec;       /* FLOCK_MATVEC_EXACT (0, the default) | FLOCK_MATVEC_FAST */
} flock_layer_config;

/* ------------------------------------------------------------- errors/dev */

/* The calling thread's last error message ("" if none). */
FLOCK_API const char* flock_last_error(void);
/* Library version string, e.g. "flock_b200 0.1 sm_100a". */
FLOCK_API const char* flock_version(void);

/* kernels/lib.ts:385 getDevice(): open GPU `ordinal` with its own stream. */
FLOCK_API int flock_dev_open(int ordinal, flock_dev** out);
FLOCK_API int flock_dev_close(flock_dev* dev);
/* Wait for all work queued on the device handle's stream. */
FLOCK_API int flock_dev_sync(flock_dev* dev);
/* Number of SMs, for launch planning by callers. */
FLOCK_API int flock_dev_sm_count(flock_dev* dev, int* out);
/* Device-event timing around the handle's stream: start, stop, elapsed ms. */
FLOCK_API int flock_dev_timer_start(flock_dev* dev);
FLOCK_API int flock_dev_timer_stop(flock_dev* dev, float* ms);

/* --------------------------------------------------------------- repack */

/* kernels/lib.ts:126 splitQ8: 34-byte blocks -> qs [rows*cols] + scales
 * [rows*cols/32*2], byte for byte.  Pure host code, no device needed. */
FLOCK_API int flock_repack_q8(const uint8_t* packed, int64_t rows, int64_t cols, uint8_t* qs_out,
                    uint8_t* scales_out);
/* kernels/lib.ts:142 splitQ4: 18-byte blocks -> qs [rows*cols/2] + scales. */
FLOCK_API int flock_repack_q4(const uint8_t* packed, int64_t rows, int64_t cols, uint8_t* qs_out,
                    uint8_t* scales_out);
/* kernels/lib.ts:94 quantMatrixQ8 (each row as lib.ts:40 quantRowQ8): f32
 * [rows][cols] -> Q8_0 blocks [rows*cols/32][34] on the host; cols a multiple
 * of 32.  Per block d = amax/127 in f64, the scale is f32(d) rounded to f16
 * (nearest even), q = round-half-up(x/d) clamped to [-128, 127]. */
FLOCK_API int flock_quant_q8(const float* w, int64_t rows, int64_t cols, uint8_t* out);
/* kernels/lib.ts:103 quantMatrixQ4 (rows as lib.ts:64 quantRowQ4): d = the
 * first value of largest magnitude / -8, q = clamp(floor(x/d + 8.5), 0, 15),
 * byte i = q[i] | q[i+16] << 4. */
FLOCK_API int flock_quant_q4(const float* w, int64_t rows, int64_t cols, uint8_t* out);

/* -------------------------------------------------------------- tensors */

/* kernels/layer.ts:289 Layer.create's per-tensor path: split the packed GGUF
 * blocks on the host and upload (dtype FLOCK_Q8_0 or FLOCK_Q4_0). */
FLOCK_API int flock_tensor_from_packed(flock_dev* dev, int dtype, const uint8_t* packed, int64_t rows,
                             int64_t cols, flock_tensor** out);
/* web/js/gguf-stream.mjs:281 streamTensorToGPU / layer.ts:73 GpuTensor
 * {qs, scales}: upload planes that are already split (fromBuffers path). */
FLOCK_API int flock_tensor_from_split(flock_dev* dev, int dtype, const uint8_t* qs, const uint8_t* scales,
                            int64_t rows, int64_t cols, flock_tensor** out);
/* layer.ts:73 GpuTensor {data}: an f32 tensor (norm gains). */
FLOCK_API int flock_tensor_from_f32(flock_dev* dev, const float* data, int64_t n, flock_tensor** out);
FLOCK_API int flock_tensor_free(flock_tensor* t);
/* Bytes resident on the device for the tensor (qs + scales, or data). */
FLOCK_API int flock_tensor_bytes(const flock_tensor* t, int64_t* out);
/* kernels/lib.ts:548 storageBuffer / :569 uniformBuffer: a raw device buffer
 * of `bytes` (rounded up to 4) holding a copy of `data` (NULL: zeros), typed
 * FLOCK_F32 so the ops that take an f32 tensor accept it. */
FLOCK_API int flock_tensor_from_bytes(flock_dev* dev, const void* data, int64_t bytes,
                                      flock_tensor** out);
/* kernels/lib.ts:576 readBack: copy [offset, offset+bytes) of an f32/raw
 * tensor's device buffer to the host (synchronous). */
FLOCK_API int flock_tensor_read(const flock_tensor* t, int64_t offset, int64_t bytes, void* out);

/* ---------------------------------------------------- op-level kernels
 * The individually validated kernels, with host inputs/outputs, as the
 * reference's kernel tests drive them (kernels/test_coop.ts, test_ops.ts,
 * test_head.ts, test_prefill.ts). */

/* kernels/q8_coop.wgsl:76 / q4_coop.wgsl:48: out[t][r] = W x[t] for n_tokens
 * rows of x ([n_tokens][cols] -> [n_tokens][rows]). */
FLOCK_API int flock_op_matvec(flock_dev* dev, const flock_tensor* w, const float* x, int n_tokens,
                    float* out);
/* Device-resident timing of the matvec (bench.ts:195 timeBatched's role):
 * `iters` back-to-back launches on a seeded device x, CUDA-event timed;
 * writes the mean milliseconds per launch. */
FLOCK_API int flock_op_matvec_timed(flock_dev* dev, const flock_tensor* w, int n_tokens, int iters,
                                    float* ms_per_call);
/* The same launch timed cold: before each of the `iters` launches a 256 MiB
 * device write evicts L2 (126 MB), so the weights stream from HBM; each
 * launch is CUDA-event timed alone; writes the mean milliseconds.  (A
 * measurement aid like bench.ts:195; allocates its scratch.) */
FLOCK_API int flock_op_matvec_timed_cold(flock_dev* dev, const flock_tensor* w, int n_tokens,
                                         int iters, float* ms_per_call);
/* The FLOCK_MATVEC_FAST matvec of one token (int8 tensor cores; the same
 * rows as flock_op_matvec to max relative error 1e-3), and its device-resident
 * timing (cold: L2 evicted before each launch, as flock_op_matvec_timed_cold).
 * Replaces nothing in the reference: its matvecs have one (the f32) order. */
FLOCK_API int flock_op_matvec_fast(flock_dev* dev, const flock_tensor* w, const float* x,
                                   float* out);
FLOCK_API int flock_op_matvec_fast_timed(flock_dev* dev, const flock_tensor* w, int iters,
                                         int cold, float* ms_per_call);
/* The prefill matmul of layer.ts:685 encodePrefill (q8_coop.wgsl:76 /
 * q4_coop.wgsl:48 over M tokens) on the tcgen05 tensor cores: y[m][r] =
 * W x[m] with s * q and x (scaled per row by a power of two) rounded to f16
 * and f32 accumulation (the tensor-core prefill path: max relative error
 * <= 1e-2).  x is [M][cols],
 * y [M][rows]; cols must be a multiple of 64 and at most 12288. */
FLOCK_API int flock_op_gemm(flock_dev* dev, const flock_tensor* w, const float* x, int M, float* y);
/* Device-resident timing of flock_op_gemm over `iters` calls on a seeded
 * device x, CUDA events around each kernel: mean milliseconds of the GEMM
 * kernel and of the activation conversion before it. */
FLOCK_API int flock_op_gemm_timed(flock_dev* dev, const flock_tensor* w, int M, int iters,
                                  float* ms_per_call, float* ms_image);
/* flock_op_gemm_timed with L2 evicted (256 MiB device write) before each
 * call, as flock_op_matvec_timed_cold. */
FLOCK_API int flock_op_gemm_timed_cold(flock_dev* dev, const flock_tensor* w, int M, int iters,
                                       float* ms_per_call, float* ms_image);
/* One rank of an n_ranks tensor-parallel peer exchange whose peers never
 * publish (local buffers nothing writes), run `calls` times with a wait
 * limit of wait_ms, each followed by the host's error check.  *first_status
 * gets the first call's status (FLOCK_E_CUDA: the bounded wait ran out),
 * the return value the last call's (FLOCK_E_CUDA: the exchange stays failed).
 * A test of the exchange's failure detection (flock_peer.cu) that needs no
 * second GPU; no counterpart in the reference. */
FLOCK_API int flock_op_peer_exchange_lone(flock_dev* dev, int n_ranks, int64_t n, int wait_ms,
                                          int calls, int* first_status);
/* kernels/rmsnorm.wgsl:41: n_vecs vectors of width n. */
FLOCK_API int flock_op_rmsnorm(flock_dev* dev, const float* x, const float* g, int n, int n_vecs, float eps,
                     float* out);
/* kernels/rope.wgsl:50 on [n_tokens][n_heads][head_dim] at pos0 + token. */
FLOCK_API int flock_op_rope(flock_dev* dev, const float* x, int n_tokens, int n_heads, int head_dim,
                  int pos0, const float* inv_freq, int pairing, float* out);
/* kernels/elementwise.wgsl:23 swiglu / :31 add. */
FLOCK_API int flock_op_swiglu(flock_dev* dev, const float* gate, const float* up, int64_t n, float* out);
FLOCK_API int flock_op_add(flock_dev* dev, const float* a, const float* b, int64_t n, float* out);
/* kernels/attention.wgsl:58: one query per head over n_keys keys of
 * [n_keys][n_kv_heads][head_dim]; mode FLOCK_ATTN_EXACT | FLOCK_ATTN_FAST. */
FLOCK_API int flock_op_attention(flock_dev* dev, const float* q, const float* k, const float* v,
                       int n_heads, int n_kv_heads, int head_dim, int n_keys, int mode,
                       float* out);
/* kernels/attention_prefill.wgsl:75: n_queries causal queries at pos0. */
FLOCK_API int flock_op_attention_prefill(flock_dev* dev, const float* q, const float* k, const float* v,
                               int n_heads, int n_kv_heads, int head_dim, int n_queries,
                               int pos0, float* out);
/* kernels/embed.wgsl:52: gather + dequantise rows of a Q8_0 tensor. */
FLOCK_API int flock_op_embed(flock_dev* dev, const flock_tensor* table, const int32_t* ids, int n,
                   float* out);
/* kernels/argmax.wgsl:83,112: lowest index among the maxima. */
FLOCK_API int flock_op_argmax(flock_dev* dev, const float* x, int64_t n, int64_t* index, float* value);

/* No counterpart in the reference.  Greedy argmax (lowest index among the
 * maxima) over n device-resident f32 logits, for callers that cannot
 * allocate device memory: a serving framework that owns the GPU's memory,
 * a decode loop that must not call cudaMalloc (it synchronises the device),
 * an FFI caller holding only raw device pointers.  x, index_out and
 * value_out are device pointers; stream may be NULL (the default stream).
 * Nothing is allocated: the per-CTA partials live in a fixed 8.25 KiB
 * device array inside the library, present on every GPU that loads it
 * until exit.  n must be <= 4194304 (FLOCK_E_LIMIT otherwise), a bound
 * this entry point chooses -- the kernel walks any n with a grid stride.
 * Every call asks the runtime for the array's address in the current
 * context, so a device reset between calls is safe; the first call on a
 * device loads the module, so make it before any stream capture.  Calls
 * share the array: calls whose kernels overlap on the GPU race, so order
 * them on one stream. */
FLOCK_API int flock_argmax_noalloc(const float* x, int64_t n, int32_t* index_out, float* value_out,
                                   void* stream);

/* ---------------------------------------------------------------- layer */

/* kernels/layer.ts:228 Layer.fromBuffers: `names` are the GGUF suffixes
 * ("attn_q.weight", ..., "ffn_norm.weight"); the layer borrows the tensors
 * (they must outlive it).  Missing tensors -> FLOCK_E_MISSING naming them. */
FLOCK_API int flock_layer_create(flock_dev* dev, const flock_layer_config* cfg, int n_tensors,
                       const char* const* names, flock_tensor* const* tensors,
                       flock_layer** out);
FLOCK_API int flock_layer_free(flock_layer* layer);
/* kernels/layer.ts:571 encode (n_tokens == 1) / :685 encodePrefill
 * (n_tokens > 1): consume `hidden` ([n_tokens][hidden]; NULL = the previous
 * output, already on the device), append n_tokens keys, leave the output on
 * the device.  Throws-equivalents: KV full, maxPrefill exceeded. */
FLOCK_API int flock_layer_encode(flock_layer* layer, const float* hidden, int n_tokens);
/* kernels/layer.ts:801 readOutput(nTokens). */
FLOCK_API int flock_layer_read_output(flock_layer* layer, int n_tokens, float* out);
/* kernels/layer.ts:451 reset(); Layer.nKeys. */
FLOCK_API int flock_layer_reset(flock_layer* layer);
FLOCK_API int flock_layer_n_keys(const flock_layer* layer, int* out);
/* Drop the cache back to n_keys (model.ts:529 rewind, per layer). */
FLOCK_API int flock_layer_rewind(flock_layer* layer, int n_keys);
/* kernels/layer.ts:792 cacheBuffers(): copy keys/values [n_keys][nKV][hd] as f32
 * (a bf16 cache is widened exactly). */
FLOCK_API int flock_layer_read_cache(flock_layer* layer, float* k_out, float* v_out);
/* Preload keys/values at the current position (a synthetic cache); a bf16
 * cache stores them rounded to nearest even. */
FLOCK_API int flock_layer_write_cache(flock_layer* layer, const float* k, const float* v, int n_keys);

/* web/bird.html:544-620 runFrame / tools/sim_bird.mjs:326-340: run `x`
 * ([seq][hidden]) through `n_layers` held layers in order at cache offset
 * `offset` (checked against every layer's nKeys unless `reset`, which
 * clears the caches first, wire.mjs FLAG_RESET), write [seq][hidden]. */
FLOCK_API int flock_range_forward(flock_layer* const* layers, int n_layers, const float* x, int seq,
                        int offset, int reset, float* out);

/* ---------------------------------------------------------------- model */

/* kernels/model.ts:109 Model.create(dev, m, cfg, {cut}): `layer_tensors` is
 * n_layers * 11 tensors in the order attn_q, attn_k, attn_v, attn_output,
 * ffn_gate, ffn_up, ffn_down, attn_norm, attn_q_norm, attn_k_norm,
 * ffn_norm; `embd` the tied [vocab][hidden] Q8_0 table; `output` the untied
 * lm-head or NULL (tied).  Holds layers 0..cut-1 (cut < 0: all). */
FLOCK_API int flock_model_create(flock_dev* dev, const flock_layer_config* cfg, int vocab, int n_layers,
                       flock_tensor* const* layer_tensors, const flock_tensor* embd,
                       const flock_tensor* output_norm, const flock_tensor* output, int cut,
                       flock_model** out);
/* One rank of a tensor-parallel model over `comm` (one rank per GPU, NCCL;
 * no counterpart in the reference, which validates shard.ts on one device).
 * The layers are this rank's slices in the shard.ts directions: `cfg` is the
 * rank-local shape (n_heads, n_kv_heads and ffn divided among the ranks),
 * attn_q/k/v, ffn_gate/up carry the rank's output rows ("row" shards),
 * attn_output and ffn_down its input columns ("col" shards), whose partial
 * products are all-gathered and summed in rank order (shardReduceRef) before
 * the residual add.  `embd` and output_norm are whole on every rank;
 * `output_slice` is the rank's rows shardRanges(vocab, n_ranks, 1)[rank] of
 * the lm-head (of embd when tied); each rank's (value, index) maximum is
 * all-gathered and reduced by reduceShardArgmax.  Every step, logits and
 * head call is a collective: all ranks make it with the same arguments.
 * Both prefill paths shard the same way; the persistent decode kernel is not
 * used (single-token steps replay the kernel graph, NCCL included). */
FLOCK_API int flock_model_create_tp(flock_dev* dev, const flock_layer_config* cfg, int vocab,
                                   int n_layers, flock_tensor* const* layer_tensors,
                                   const flock_tensor* embd, const flock_tensor* output_norm,
                                   const flock_tensor* output_slice, flock_comm* comm,
                                   flock_model** out);
/* How a tensor-parallel model's decode steps exchange the o_proj / down
 * partials: FLOCK_TP_PEER (default when every rank can map every peer's
 * memory) -- one kernel per exchange pushes this rank's partial into every
 * rank's buffer over NVLink, publishes an epoch flag and sums the ranks'
 * partials in rank order once all flags arrived (bounded wait); or
 * FLOCK_TP_NCCL -- an NCCL all-gather and the same ordered sum.  Both give
 * identical bits.  Multi-token steps always use NCCL. */
#define FLOCK_TP_NCCL 0
#define FLOCK_TP_PEER 1
FLOCK_API int flock_model_set_tp_exchange(flock_model* m, int mode);
FLOCK_API int flock_model_get_tp_exchange(const flock_model* m, int* mode);
FLOCK_API int flock_model_free(flock_model* m);
/* kernels/model.ts:387 step(ids): prefill/decode ids, return the greedy id. */
FLOCK_API int flock_model_step(flock_model* m, const int32_t* ids, int n, int32_t* next_id);
/* kernels/model.ts:400 logits(ids): the [vocab] logits of the last position. */
FLOCK_API int flock_model_logits(flock_model* m, const int32_t* ids, int n, float* logits);
/* kernels/model.ts:409 hiddenState / :491 normedState. */
FLOCK_API int flock_model_hidden_state(flock_model* m, const int32_t* ids, int n, float* out);
FLOCK_API int flock_model_normed_state(flock_model* m, const int32_t* ids, int n, float* out);
/* kernels/model.ts:546 embed(ids). */
FLOCK_API int flock_model_embed(flock_model* m, const int32_t* ids, int n, float* out);
/* kernels/model.ts:437 encodePartial(ids, offset): [n][hidden] after the held
 * layers; offset < 0 skips the check. */
FLOCK_API int flock_model_encode_partial(flock_model* m, const int32_t* ids, int n, int offset, float* out);
/* kernels/model.ts:474 projectHidden(flat, seq): head on the last row. */
FLOCK_API int flock_model_project_hidden(flock_model* m, const float* flat, int seq, int32_t* next_id);
/* kernels/model.ts:572 generate(prompt, maxTokens, {eos}): host loop of
 * step(), one 4-byte readback per token, stopping at an eos id. */
FLOCK_API int flock_model_generate(flock_model* m, const int32_t* prompt, int n_prompt, int max_tokens,
                         const int32_t* eos, int n_eos, int32_t* out_ids, int* n_out);
/* Greedy decode with the token fed back on the device (no per-token host
 * round trip): `n_steps` decode steps from the token the last step chose,
 * replayed from one captured CUDA graph; ids are read back at the end. */
FLOCK_API int flock_model_decode_device(flock_model* m, int n_steps, int32_t* out_ids);
/* kernels/model.ts:199 reset() / :529 rewind(nKeys) / pos / held. */
FLOCK_API int flock_model_reset(flock_model* m);
FLOCK_API int flock_model_rewind(flock_model* m, int n_keys);
FLOCK_API int flock_model_pos(const flock_model* m, int* out);
FLOCK_API int flock_model_held(const flock_model* m, int* out);
#define FLOCK_DECODE_KERNELS 0    /* one kernel per op, CUDA graph + PDL */
#define FLOCK_DECODE_PERSISTENT 1 /* one cooperative persistent kernel per token */
#define FLOCK_DECODE_EAGER 2      /* one kernel per op, launched from the host each step */
#define FLOCK_DECODE_STREAM 3     /* one cooperative kernel per token, weights streamed
                                     through shared-memory rings */
/* Choose the decode engine for single-token steps (default: the kernel
 * graph).  The persistent and streaming kernels need fast attention, Q8_0
 * weights, head_dim 128, a GQA group of at most 4 and a whole single-GPU
 * model with its embedding/head; otherwise the kernel graph runs and
 * flock_model_get_decode_mode reports it.  The persistent kernel is
 * bit-identical to the graph; the streaming kernel's matvecs are too (same
 * coop(64) order), its split-K attention uses 32-key splits (a different
 * reassociation of the softmax, within the same tolerance of attnRef). */
FLOCK_API int flock_model_set_decode_mode(flock_model* m, int mode);
FLOCK_API int flock_model_get_decode_mode(const flock_model* m, int* mode);
/* Phase trace of the persistent decode kernel (a profiling aid with no
 * counterpart in the reference): while enabled, each CTA records 10 + 10 * held
 * global-timer nanosecond values per token -- stamps at start, embedded, then
 * for every layer and each of its 5 phases (QKV, attention, o_proj, gate/up,
 * down) "computed" and "released by the grid barrier", head computed and
 * done; then 6 words kept zero.  trace_read copies the last token's
 * [n_ctas][stride] entries. */
FLOCK_API int flock_model_trace(flock_model* m, int enable);
FLOCK_API int flock_model_trace_read(flock_model* m, uint64_t* out, int64_t cap, int* n_ctas,
                                     int* stride);
/* Set the token the next device-fed decode step consumes (ids[0]). */
FLOCK_API int flock_model_set_token(flock_model* m, int32_t id);
/* kernels/model.ts:541 currentToken(). */
FLOCK_API int flock_model_current_token(flock_model* m, int32_t* out);

/* ------------------------------------------------------------ FLK1 frames */

/* web/js/wire.mjs FLK1 frames: "FLK1" | seq | hidden | offset | flags (u32 LE,
 * flags bit 0 reset, bit 1 replay) | f16 payload.  pack (wire.mjs:54) rounds
 * f32 to f16 to nearest even (subnormals, overflow to inf, NaN -> 0x7e00 |
 * sign) and needs 20 + 2n bytes (*out_len, FLOCK_E_LIMIT if cap is short);
 * unpack (wire.mjs:79) widens exactly (NaN canonical) and fills meta = {seq,
 * hidden, offset, reset, replay}; out == NULL reads the header only. */
FLOCK_API int flock_wire_pack(const float* x, int64_t n, uint32_t seq, uint32_t hidden,
                              uint32_t offset, uint32_t flags, uint8_t* out, int64_t cap,
                              int64_t* out_len);
FLOCK_API int flock_wire_unpack(const uint8_t* frame, int64_t len, float* out, int64_t cap,
                                uint32_t meta[5]);
/* web/bird.html:544 runFrame for a held layer range: the frame's f16 payload is
 * widened on the device, a reset flag clears the caches first, the offset must
 * equal the caches' position ("cache holds X positions, frame is at Y"), the
 * layers run in order and the output frame (same header) carries the last
 * layer's output rounded to f16 as pack() would. */
FLOCK_API int flock_range_forward_wire(flock_layer* const* layers, int n_layers,
                                       const uint8_t* frame, int64_t frame_len, uint8_t* out,
                                       int64_t out_cap, int64_t* out_len);

/* ----------------------------------------------------------------- GGUF */

/* A GGUF model file opened on the host (web/js/gguf-dir.mjs:187
 * readDirectory / server/gguf.mjs:48 readModel): the directory is parsed at
 * open (version 2 or 3; dataStart = header end rounded up to
 * general.alignment, default 32); tensor bytes are read on demand. */
typedef struct flock_gguf flock_gguf;
FLOCK_API int flock_gguf_open(const char* path, flock_gguf** out);
FLOCK_API int flock_gguf_free(flock_gguf* g);
/* tensor count, dataStart, version, `<general.architecture>.block_count` (-1 if absent) */
FLOCK_API int flock_gguf_info(const flock_gguf* g, int64_t* n_tensors, int64_t* data_start,
                              int* version, int* n_layers);
/* tensor i: name (NUL-terminated, cut to name_cap), ggml type (0 F32, 1 F16,
 * 2 Q4_0, 8 Q8_0, ...), rows (product of shape[1:]), cols (shape[0]; GGUF
 * shapes are [in, out]), offset from dataStart, bytes (gguf.mjs:37
 * tensorBytes; -1 for a type without block geometry). */
FLOCK_API int flock_gguf_tensor_info(const flock_gguf* g, int64_t i, char* name, int name_cap,
                                     int* dtype, int64_t* rows, int64_t* cols, int64_t* offset,
                                     int64_t* bytes);
FLOCK_API int flock_gguf_find(const flock_gguf* g, const char* name, int64_t* index);
/* metadata by key: integers and bools (arrays: their length), numbers, strings */
FLOCK_API int flock_gguf_meta_int(const flock_gguf* g, const char* key, int64_t* out);
FLOCK_API int flock_gguf_meta_f64(const flock_gguf* g, const char* key, double* out);
FLOCK_API int flock_gguf_meta_str(const flock_gguf* g, const char* key, char* out, int cap);
/* server/gguf.mjs:78 byteRanges: absolute byte ranges covering the blk.<first..last>.*
 * tensors, merged where the gap is at most `gap` bytes; *n = the count
 * (FLOCK_E_LIMIT when it exceeds cap). */
FLOCK_API int flock_gguf_layer_ranges(const flock_gguf* g, int first, int last, int64_t gap,
                                      int64_t* starts, int64_t* ends, int cap, int* n);
/* web/js/gguf-stream.mjs:281 streamTensorToGPU: the tensor's bytes read
 * `staging` bytes at a time (<= 0: 4 MiB), Q8_0 / Q4_0 blocks split into the
 * qs and scale planes as they arrive (SplitStreamer, :132) and copied to the
 * device from two pinned staging buffers in turn; F32 / F16 tensors (norm
 * gains) become f32 data. */
FLOCK_API int flock_gguf_load_tensor(flock_dev* dev, const flock_gguf* g, const char* name,
                                     int64_t staging, flock_tensor** out);
/* The same incremental split into host planes in block order (qs: 32 / 16
 * bytes per block, scales: 2), reading `chunk` bytes at a time. */
FLOCK_API int flock_gguf_split_host(const flock_gguf* g, const char* name, int64_t chunk,
                                    uint8_t* qs, uint8_t* scales);

/* --------------------------------------------------------------- shards */

/* kernels/shard.ts:214 ShardedMatvec.create over a Q8_0 tensor given in the
 * split layout ([rows][cols] qs + scales), direction 0 = row (output-split),
 * 1 = col (input-split); binding_limit <= 0 means no limit.  All shards live
 * on `dev` (the reference's single-device validation form). */
FLOCK_API int flock_shard_matvec_create(flock_dev* dev, const uint8_t* qs, const uint8_t* scales,
                              int64_t rows, int64_t cols, int n_shards, int direction,
                              int64_t binding_limit, flock_shard** out);
FLOCK_API int flock_shard_matvec_free(flock_shard* s);
/* shard.ts:320 setInput + :340 encode + :400 output: y = W x. */
FLOCK_API int flock_shard_matvec_run(flock_shard* s, const float* x, float* y);
/* shard.ts:405 partials(): [n_shards][rows] (col direction only). */
FLOCK_API int flock_shard_matvec_partials(flock_shard* s, float* parts);
/* shard.ts:411 wireBytesPerCall(). */
FLOCK_API int flock_shard_matvec_wire_bytes(const flock_shard* s, int64_t* out);

/* kernels/shard.ts:502 ShardedHead.create: row-sharded LM head with
 * per-shard argmax and the cross-shard reduce (shard_ref.ts:437). */
FLOCK_API int flock_sharded_head_create(flock_dev* dev, const uint8_t* qs, const uint8_t* scales,
                              int64_t vocab, int64_t hidden, int n_shards, flock_head** out);
FLOCK_API int flock_sharded_head_free(flock_head* h);
/* shard.ts:582 setInput + :595 encode: logits [vocab] (optional) and token. */
FLOCK_API int flock_sharded_head_run(flock_head* h, const float* x, float* logits, int32_t* token);
/* shard.ts:632 argmaxBuffers(): per-shard (value, local index, row offset). */
FLOCK_API int flock_sharded_head_shard_argmax(flock_head* h, float* values, int64_t* index,
                                    int64_t* row_offset);

/* ------------------------------------------------- multi-GPU (NCCL) */

/* NCCL unique id (128 bytes) for rank 0 to broadcast to the others. */
FLOCK_API int flock_comm_unique_id(uint8_t id_out[128]);
/* One communicator per process/GPU; timeout_ms bounds every collective. */
FLOCK_API int flock_comm_init(flock_dev* dev, int n_ranks, int rank, const uint8_t id[128], int timeout_ms,
                    flock_comm** out);
FLOCK_API int flock_comm_free(flock_comm* c);
/* Pipeline hop (replaces server/mesh.js:679 Flock.lap's wire hop): send /
 * receive `n` f32 of device-resident hidden state to/from `peer`. */
FLOCK_API int flock_comm_send_hidden(flock_comm* c, flock_model* m, int n_tokens, int peer);
FLOCK_API int flock_comm_recv_hidden(flock_comm* c, flock_model* m, int n_tokens, int peer);
/* One pipeline step on this rank (kernels/model.ts encodeTokens + encodeHead
 * split across ranks, server/mesh.js:679 lap): rank 0 embeds `ids` (NULL =
 * the id its head chose last step, already on the device), runs its layers,
 * sends the hidden state on, receives it back from the last rank and runs
 * the head; rank r > 0 receives, runs its layer range and sends on.  With
 * sync = 0 nothing waits on the host (a device-resident decode loop).  A
 * NULL communicator is the single-GPU case. */
FLOCK_API int flock_pipeline_step(flock_model* m, flock_comm* c, const int32_t* ids, int n,
                                  int sync, int32_t* next_id);
/* Token ids the head chose at positions [start, start+n) (rank 0). */
FLOCK_API int flock_model_history(flock_model* m, int start, int n, int32_t* out);
/* Host-buffer all-reduce (sum, f32) and all-gather, for tests and planners. */
FLOCK_API int flock_comm_allreduce_f32(flock_comm* c, const float* in, float* out, int64_t n);
FLOCK_API int flock_comm_allgather_bytes(flock_comm* c, const void* in, void* out, int64_t bytes_per_rank);

#ifdef __cplusplus
}
#endif
#endif /* FLOCK_CUDA_H */
