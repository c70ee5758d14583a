/* TEST INFRASTRUCTURE ONLY -- the parity checker, never shipped or measured as the product.
 *
 * Plain-C restatement of the reference decode path (astrowar/MiniCPM5.cpp).
 * Every function names the reference code it restates.  Block layouts are the
 * reference's byte layouts (include/ops.h:33-65).
 */
#ifndef MCPM_ORACLE_H
#define MCPM_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ORC_QK_K 256
#define ORC_QK8_0 32
enum { ORC_F32 = 0, ORC_Q8_0 = 8, ORC_Q4_K = 12, ORC_Q6_K = 14 };
enum { ORC_ROUND_EVEN = 0, ORC_ROUND_AWAY = 1 };
enum { ORC_ORDER_SCALAR = 0, ORC_ORDER_AVX2 = 1, ORC_ORDER_BATCH = 2 };

float orc_fp16_to_fp32(uint16_t h);
void orc_q4k_scales_mins(const uint8_t q[12], uint8_t sc[8], uint8_t mn[8]);

/* fp32 -> block_q8_K (292 B per 256).  rounding: ORC_ROUND_EVEN follows
 * quantize_row_q8_K_avx2 / _scalar, ORC_ROUND_AWAY follows the lround of the fused
 * norm / SwiGLU quantisers.  recip_d: d = amax * (1/127) instead of amax / 127. */
void orc_quantize_q8k(const float* x, int n, void* y, int rounding, int recip_d);

/* Integer block sums (exact).  q4k: isum = sum_j sc[j]*dot_j, minsum = sum_g mn[g]*(bs[2g]+bs[2g+1]).
 * q6k: isum = sum over unsigned q in [0,63] of sc*q*x, offset = 32*sum_g sc[g]*bsums[g]. */
void orc_q4k_block_sums(const void* wblk, const void* xblk, int32_t* isum, int32_t* minsum);
void orc_q6k_block_sums(const void* wblk, const void* xblk, int32_t* isum, int32_t* offset);
/* Whole-matrix block sums, [rows][nb] each. */
void orc_blocksums(int type, const void* w, const void* xq, int rows, int cols, int32_t* isum, int32_t* aux);

/* GEMV over a pre-quantised Q8_K activation.  order selects the fp32 accumulation order:
 * ORC_ORDER_SCALAR follows dot_row_q*_K_q8_K_scalar, ORC_ORDER_AVX2 the eight-lane
 * accumulators + horizontal sum of dot_row_q*_K_q8_K_avx2 (the batch-1 decode kernel),
 * ORC_ORDER_BATCH the tcgen05 batched GEMM's order: the exact block sum isum (Q6_K: minus its
 * -32 offset) scaled by one fma per block, acc = fma(xd*d, isum, acc) and (Q4_K)
 * accm = fma(-(xd*dmin), minsum, accm) over groups of 4 consecutive blocks, g = acc + accm per
 * group, row = ((g0 + g1) + g2) + ... .  fused_min: contract the Q4_K min term into one fused
 * multiply-subtract (AVX2 order). */
void orc_gemv_q4k_q8k(const void* w, const void* xq, float* y, int rows, int cols, int order, int fused_min);
void orc_gemv_q6k_q8k(const void* w, const void* xq, float* y, int rows, int cols, int order);
/* gemv_q8_0 (src/ops/ops.cpp:58-79): fp32 activations, per-32 sum then * fp16(d). */
void orc_gemv_q8_0(const void* w, const float* x, float* y, int rows, int cols);

/* Canonical numerics shared with the CUDA kernels (see mcpm_oracle.c for each order). */
float orc_sumsq(const float* x, int n);
float orc_rms_scale(const float* x, int n, float eps);
float orc_expf(float x);
float orc_block_amax(const float* y);
float orc_silu_mul(float g, float u);
void orc_rope_row(int pos, int head_dim, float base, float* cs);
int orc_attn_chunk(int n);

/* rmsnorm_and_quantize_q8k (ops.cpp:676-723). */
void orc_rmsnorm_q8k(const float* x, const float* w, int n, float eps, void* out);
/* rmsnorm (ops.cpp:468-481). */
void orc_rmsnorm(const float* x, const float* w, int n, float eps, float* out);
/* swiglu_and_quantize_q8k (ops.cpp:725-765). */
void orc_swiglu_q8k(const float* g, const float* u, int n, void* out);
/* apply_rope over n_heads heads (ops.cpp:502-516). */
void orc_rope(float* v, int n_heads, int head_dim, int pos, float base);
/* execute_attention (ops.cpp:537-628); kc/vc: [max_seq][n_kv*head_dim]. Returns 0, or -1 if pos >= max_seq. */
int orc_attention(float* out, const float* q, const float* k, const float* v, float* kc, float* vc,
                  int pos, int max_seq, int n_head, int n_kv, int head_dim);
/* get_embedding (ops.cpp:631-673) for Q4_K; Q8_0 rows are d*q. */
void orc_embedding(const void* w, int type, int token, int dim, float* out);

/* Whole-model forward (src/model.cpp:142-242). */
typedef struct {
    const uint8_t* base;                 /* file image */
    uint64_t tok_embd, out_norm, output; /* absolute offsets */
    int tok_embd_type, output_type;
    uint64_t layer[64][9];               /* attn_k attn_norm attn_output attn_q attn_v ffn_down ffn_gate ffn_norm ffn_up */
    int layer_type[64][9];
    int n_layer, n_embd, n_ff, n_head, n_head_kv, n_vocab;
    float rope_base, eps;
    int kv_f16;   /* 1: K and V rows are rounded to IEEE half precision (nearest even) as they
                     enter the cache -- the engine's fp16 KV-cache option; 0: fp32 (the reference) */
} orc_model_desc;

typedef struct orc_state orc_state;
orc_state* orc_create(const orc_model_desc* d, int max_seq);
void orc_destroy(orc_state* s);
/* Returns the greedy argmax (lowest index on ties), or -1 if pos >= max_seq. logits may be NULL. */
int orc_forward(orc_state* s, int token, int pos, float* logits);
/* GEMV order of the K-quant projections in later orc_forward calls (ORC_ORDER_AVX2, the
 * default: batch-1 decode; ORC_ORDER_BATCH: batched decode and prefill on tcgen05). */
void orc_set_order(orc_state* s, int order);
/* Copies of internal state for debugging parity: the fp32 residual x after the last call. */
void orc_get_x(const orc_state* s, float* x);
void orc_get_kv(const orc_state* s, int layer, float* k, float* v, int n_pos);
/* Overwrites rows [0, n_pos) of one layer's K/V cache (seeds a late-position check). */
void orc_set_kv(orc_state* s, int layer, const float* k, const float* v, int n_pos);

/* Top-p sampling (Sampler::sample, src/sampler.cpp:8-72) in the canonical form the device
 * sampler computes: temperature as the reference (applied only for t > 0, t != 1), max from
 * -1e9, e = orc_expf(v - max), p = e / S; order by p descending then index ascending; every
 * fp32 sum blocked over 1024 ranges of ceil(m / 1024) positions (each range sequential from
 * the running prefix of the range totals); keep the shortest prefix whose running sum reaches
 * top_p (0 < top_p < 1; otherwise all tokens in index order, not renormalised); q = p / C;
 * return the first kept token whose running sum of q is >= r, else the last kept token.
 * kept (optional) receives the number of kept tokens. */
int orc_sample_top_p(const float* logits, int n, float temperature, float top_p, float r, int* kept);

#ifdef __cplusplus
}
#endif
#endif
