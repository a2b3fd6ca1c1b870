/*
 * flock_oracle -- CPU restatement of flock's strict-f32 reference path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the parity checker for the CUDA
 * product path in flock_b200/.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py may load it; the product
 * never links, imports or falls back to it.
 *
 * What it restates (paths relative to the ethanhinson/flock project root):
 *   kernels/lib.ts       halfToF32 :30, quantRowQ8 :40, quantRowQ4 :64,
 *                        quantMatrixQ8/Q4 :94/:103, splitQ8/Q4 :126/:142,
 *                        fma32 :169, dot4 :196, matmulF32 :213,
 *                        cpuMatmulQ8F32 :251, cpuMatmulQ4F32 :280, treeSum :312
 *   kernels/ops_ref.ts   rmsnormRef :20, ropeRef :65, ropeInvFreq :95,
 *                        swigluRef :103, addRef :113, attnRef :135
 *   kernels/head_ref.ts  embedRef :34, argmaxRef :65, attnPrefillRef :99
 *   kernels/layer_ref.ts layerForwardRef :32, layerPrefillRef :103
 *   kernels/model.ts     encodeHead :307 (output_norm once, tied head, argmax)
 *   kernels/shard_ref.ts shardRanges :97, sliceRows/Cols :137/:166,
 *                        slicePacked* :196/:218, shardMatvecRef :278,
 *                        shardReduceRef :327, shardedCol/RowMatvecRef :353/:378,
 *                        reduceShardArgmax :437, memShardPlan :509
 *   kernels/dequant.ts   dequantQ8 :22, requantWithNoise :58
 *   web/js/wire.mjs      f32to16 :309, f16to32 :333, pack :344, unpack :358
 *
 * Arithmetic model.  JS numbers are IEEE f64 and Math.fround rounds to f32, so
 * every fr(...) in the reference is a (float) cast of a double here, and the
 * reference's fma32(a,b,c) = fround(a*b + c) is restated literally as
 * (float)((double)a*b + c): an exact f64 product, one f64 add, one f32 round.
 * That is a single rounding whenever a*b+c is representable in f64 (always for
 * the int8 x f32 products of the matvecs), and can differ from an IEEE fmaf by
 * one ulp on the rare f32 x f32 chains where it is not.  flock_oracle_set_fma_mode
 * switches fma32 to fmaf so a difference can be attributed to exactly that.
 * Transcendentals are (float)exp((double)x) etc., i.e. fr(Math.exp(x)).
 *
 * Build flags matter: -ffp-contract=off so the compiler never fuses a
 * restated multiply and add.
 */
#ifndef FLOCK_ORACLE_H
#define FLOCK_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* 0 = literal JS fma32 (double rounding), 1 = IEEE fmaf (single rounding). */
void fo_set_fma_mode(int mode);
int fo_get_fma_mode(void);
/* OpenMP threads for the row-parallel loops (1 = the reference's single thread). */
void fo_set_threads(int n);
int fo_max_threads(void);

/* --- codecs (lib.ts:30, wire.mjs:309,333) --- */
double fo_half_to_f32(uint16_t h);
uint16_t fo_f32to16(double v);
double fo_f16to32(uint16_t h);

/* --- quantizers and repack (lib.ts:40-156) --- */
void fo_quant_row_q8(const float* vals, int64_t n, uint8_t* out);
void fo_quant_row_q4(const float* vals, int64_t n, uint8_t* out);
void fo_quant_matrix_q8(const float* w, int64_t rows, int64_t cols, uint8_t* out);
void fo_quant_matrix_q4(const float* w, int64_t rows, int64_t cols, uint8_t* out);
void fo_split_q8(const uint8_t* packed, int64_t rows, int64_t cols, uint8_t* qs, uint8_t* scales);
void fo_split_q4(const uint8_t* packed, int64_t rows, int64_t cols, uint8_t* qs, uint8_t* scales);

/* --- matvec references (lib.ts:213-309). lanes = 0 -> SERIAL, else coop(lanes). --- */
void fo_matmul_q8(const uint8_t* packed, const float* x, int64_t rows, int64_t cols, int lanes,
                  float* out);
void fo_matmul_q4(const uint8_t* packed, const float* x, int64_t rows, int64_t cols, int lanes,
                  float* out);
/* n_tokens matvecs over [n_tokens][cols] -> [n_tokens][rows]; layer_ref.ts:335 mv(). */
void fo_matmul_q8_batched(const uint8_t* packed, const float* x, int64_t rows, int64_t cols,
                          int n_tokens, int lanes, float* out);

/* --- ops (ops_ref.ts) --- */
void fo_rmsnorm(const float* x, const float* g, int n, int n_vecs, double eps, int wg, float* out);
void fo_rope_inv_freq(int head_dim, double base, float* out);
void fo_rope(const float* x, int n_tokens, int n_heads, int head_dim, int pos0,
             const float* inv_freq, int neox, float* out);
void fo_swiglu(const float* gate, const float* up, int64_t n, float* out);
void fo_add(const float* a, const float* b, int64_t n, float* out);
void fo_attn(const float* q, const float* k, const float* v, int n_heads, int n_kv_heads,
             int head_dim, int n_keys, float* out);

/* --- head ops (head_ref.ts) --- */
void fo_embed(const uint8_t* packed, const int32_t* ids, int n_ids, int cols, float* out);
int64_t fo_argmax(const float* x, int64_t n);
void fo_attn_prefill(const float* q, const float* k, const float* v, int n_heads, int n_kv_heads,
                     int head_dim, int n_queries, int pos0, int tile, int wg, float* out);

/* --- layer (layer_ref.ts). Weights in the 34-byte packed layout. --- */
typedef struct fo_layer_cfg {
  int hidden, n_heads, n_kv_heads, head_dim, ffn;
  double eps, rope_base;
  int neox;
} fo_layer_cfg;

typedef struct fo_layer_w {
  const uint8_t* q; /* attn_q.weight      [nH*hd][hidden] */
  const uint8_t* k; /* attn_k.weight      [nKV*hd][hidden] */
  const uint8_t* v; /* attn_v.weight      [nKV*hd][hidden] */
  const uint8_t* o; /* attn_output.weight [hidden][nH*hd] */
  const uint8_t* gate, *up; /* [ffn][hidden] */
  const uint8_t* down; /* [hidden][ffn] */
  const float* attn_norm, *q_norm, *k_norm, *ffn_norm;
} fo_layer_w;

/* Reference KV cache (layer_ref.ts:24 RefCache): keys [cap][nKV*hd]. */
typedef struct fo_cache {
  float* k;
  float* v;
  int n;   /* keys held */
  int cap; /* capacity in keys */
  int kvw; /* nKV*hd */
  int bf16; /* 1: every key/value is rounded to bf16 (nearest even) as it is stored;
               2: to e4m3 (FLOCK_KV_FP8) */
} fo_cache;

fo_cache* fo_cache_new(int cap, int kvw);
void fo_cache_free(fo_cache* c);
void fo_cache_reset(fo_cache* c);
int fo_cache_len(const fo_cache* c);
const float* fo_cache_k(const fo_cache* c);
const float* fo_cache_v(const fo_cache* c);
/* A bf16 KV cache (FLOCK_KV_BF16 in flock_cuda.h; beyond the reference, which
 * keeps f32): from now on fo_cache_fill stores each value rounded to bf16. */
void fo_cache_set_bf16(fo_cache* c, int on);
/* f32 -> the nearest bf16 value (ties to even), as an f32. */
float fo_bf16_round(float x);
/* An e4m3 KV cache (FLOCK_KV_FP8): from now on fo_cache_fill stores each
 * value rounded with fo_fp8_round. */
void fo_cache_set_fp8(fo_cache* c, int on);
/* f32 -> the nearest OCP E4M3FN value (ties to even; magnitudes at or past 448
 * become 448 with the sign, NaN stays NaN), as an f32: the rounding of the
 * device's cvt.rn.satfinite.e4m3x2.f32. */
float fo_fp8_round(float x);
/* Preload n keys (e.g. a synthetic cache); returns 0 or -1 if over capacity. */
int fo_cache_fill(fo_cache* c, const float* k, const float* v, int n);

/* layerForwardRef (n_tokens == 1) / layerPrefillRef (n_tokens > 1). Returns 0 or -1. */
int fo_layer_forward(const float* hidden, const fo_layer_w* w, const fo_layer_cfg* cfg,
                     fo_cache* cache, float* out);
int fo_layer_prefill(const float* hidden, int n_tokens, const fo_layer_w* w,
                     const fo_layer_cfg* cfg, fo_cache* cache, float* out);
/* The tensor-parallel layer: o_proj and down as tp-shard input-split matvecs
 * (shardedColMatvecRef); tp == 1 is fo_layer_prefill. */
int fo_layer_prefill_tp(const float* hidden, int n_tokens, const fo_layer_w* w,
                        const fo_layer_cfg* cfg, fo_cache* cache, int tp, float* out);

/* model.ts encodeHead :307: rmsnorm(output_norm) -> tied head coop(64) -> argmax. */
int64_t fo_head(const float* last_row, const float* out_norm, const uint8_t* embd_packed,
                int64_t vocab, int hidden, double eps, float* normed_out, float* logits_out);

/* --- shard_ref.ts --- */
/* Fills starts/counts (length n); returns 0, or -1 (bad arg), -2 (not multiple of align),
 * -3 (fewer units than shards).  shard_ref.ts:97. */
int fo_shard_ranges(int64_t total, int n, int64_t align, int64_t* starts, int64_t* counts);
void fo_slice_rows(const uint8_t* qs, const uint8_t* scales, int64_t rows, int64_t cols,
                   int64_t start, int64_t end, uint8_t* qs_out, uint8_t* sc_out);
int fo_slice_cols(const uint8_t* qs, const uint8_t* scales, int64_t rows, int64_t cols,
                  int64_t start, int64_t end, uint8_t* qs_out, uint8_t* sc_out);
int fo_slice_packed_cols(const uint8_t* packed, int64_t rows, int64_t cols, int64_t start,
                         int64_t end, uint8_t* out);
void fo_shard_matvec(const uint8_t* packed, const float* x, int64_t rows, int64_t cols, int lanes,
                     float* out);
void fo_shard_reduce(const float* parts, int n_shards, int64_t n, float* out);
int fo_sharded_col_matvec(const uint8_t* packed, const float* x, int64_t rows, int64_t cols,
                          int n_shards, int lanes, float* out);
int fo_sharded_row_matvec(const uint8_t* packed, const float* x, int64_t rows, int64_t cols,
                          int n_shards, int lanes, float* out);
int64_t fo_reduce_shard_argmax(const float* values, const int64_t* index,
                               const int64_t* row_offset, int n);
/* memShardPlan: fills max binding bytes of the plan, the unsharded figure and
 * the minimum shard count (0 = none fits).  dir 0 = row, 1 = col. */
int fo_mem_shard_plan(int64_t rows, int64_t cols, double bytes_per_weight,
                      double scale_bytes_per_block, int n, int dir, double limit,
                      double* max_binding, double* unsharded, int64_t* min_shards, int* fits);

/* --- dequant.ts --- */
void fo_dequant_q8(const uint8_t* packed, int64_t rows, int64_t cols, float* out);
/* One tensor of requantWithNoise; `state` carries xorshift32 across tensors. */
void fo_requant_with_noise(const uint8_t* packed, int64_t rows, int64_t cols, uint32_t* state,
                           uint8_t* out);

/* --- wire.mjs FLK1 frame --- */
int64_t fo_wire_pack(const float* floats, int64_t n, uint32_t seq, uint32_t hidden,
                     uint32_t offset, int reset, int replay, uint8_t* out);
int fo_wire_unpack(const uint8_t* buf, int64_t nbytes, float* out, uint32_t* meta5);

#ifdef __cplusplus
}
#endif
#endif
