/*
 * CPU oracle for the LeanInfer fused-kernel path. TEST INFRASTRUCTURE ONLY:
 * it is the checker the CUDA kernels are compared against, and the timed
 * CPU baseline of bench.py. No product code links or calls it.
 *
 * Every function restates the reference's arithmetic (file:line cited at
 * each definition in li_oracle.c) in double precision, except the block
 * decoders, which reproduce gguf-py's fp32 arithmetic bit for bit.
 */
#pragma once
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

float  lio_fp16_to_fp32(uint16_t h);
float  lio_bf16_to_fp32(uint16_t h);
uint16_t lio_fp32_to_bf16(float f);          /* round to nearest even */
size_t lio_row_bytes(int wtype, int64_t k);

/* Block decode (ggml to_float). n values. */
int lio_dequantize(int wtype, const void *src, float *dst, int64_t n);

/* dst[r][n] = <rmsnorm(x[r])*gamma or x[r], W[n]>; gamma NULL = no norm. */
int lio_rms_norm_matmul(int wtype, const float *x, const float *gamma,
                        const void *W, float *dst, int K, int N, int n_rows,
                        float eps);

/* The same with ggml-style quantized activations (q8_K for Q4_K weights,
 * q8_0 for Q8_0) and integer dots; UNPINNED (no reference vector fixes
 * ggml's CPU results): a measure of that arithmetic's distance from the
 * exact dots, not a parity target. */
int lio_rms_norm_matmul_q8act(int wtype, const float *x, const float *gamma,
                              const void *W, float *dst, int K, int N,
                              int n_rows, float eps);

/* h[r][n] = silu(<xn, Wg[n]>) * <xn, Wu[n]>. round_xn_f16 rounds xn to fp16
 * before the dots (the reference f16 kernel's behaviour). */
int lio_rms_norm_swiglu(int wtype, const float *x, const float *gamma,
                        const void *Wg, const void *Wu, float *h, int K, int N,
                        int n_rows, float eps, int round_xn_f16);

/* y = Wd . swiglu(x) with Wd [K, N]. */
int lio_ffn(int wtype, const float *x, const float *gamma, const void *Wg,
            const void *Wu, const void *Wd, float *y, int K, int N, int n_rows,
            float eps);

/* dst[r][k] = silu(z[r][k]) * o[r][k] * gamma[k] * rsqrt(mean(o[r]^2)+eps). */
void lio_silu_gate(const float *o, const float *z, const float *gamma,
                   float *dst, int K, int n_rows, float eps);

/* Reference-layout recurrence; see include/leaninfer-cuda.h. proj_out may be
 * NULL; W_out fp32 [hidden, n_heads*D]. */
int lio_deltanet_recurrent(const float *q, const float *k, const float *v,
                           const float *g, const float *beta,
                           const float *state_in, float *out, float *state_out,
                           const float *W_out, float *proj_out,
                           int64_t D, int64_t n_tokens, int64_t n_heads,
                           int64_t gqa, int repeat_type, int64_t n_seqs,
                           int64_t hidden, size_t vnb1, size_t vnb2,
                           size_t vnb3);

typedef struct lio_deltanet_layer {
    int hidden, n_k_heads, n_v_heads, head_dim, conv_kernel, repeat_type;
    int w_in_type, w_out_type;
    float in_norm_eps, norm_eps, l2_eps;
    const float *in_norm_w;
    const void *w_in;
    const float *conv_w, *a_log, *dt_bias, *norm_w;
    const void *w_out;
} lio_deltanet_layer;

/* One decode step of a DeltaNet layer for n_seqs sequences; conv_state and
 * state updated in place. If taps is non-NULL it receives, per sequence and
 * back to back: the post-conv activations (q|k|v, 2*Hk*D + Hv*D), z (Hv*D),
 * beta (Hv), g (Hv), o (Hv*D) and the gated o (Hv*D). */
size_t lio_deltanet_taps_per_seq(const lio_deltanet_layer *L);
int lio_deltanet_layer_decode(const lio_deltanet_layer *L, const float *x,
                              float *y, float *conv_state, float *state,
                              int n_seqs, float *taps);

/* The same step with the projections in ggml's CPU arithmetic (quantized
 * activations, integer dots); UNPINNED, the timed CPU baseline's form. */
int lio_deltanet_layer_decode_q8act(const lio_deltanet_layer *L, const float *x,
                                    float *y, float *conv_state, float *state,
                                    int n_seqs);

/* Sequential gated delta rule over T tokens, one sequence, in the token-major
 * layout of the prefill entry: q, k bf16 (as uint16) [T, Hk, D]; v bf16
 * [T, Hv, D]; g, beta fp32 [T, Hv] (beta already a probability, g the
 * log-decay); v-head h reads k-head h / (Hv/Hk). state [Hv][D(k)][D(v)] fp32
 * in/out; o fp32 [T, Hv, D]. No clamp: the plain gated delta rule. */
int lio_gdr_prefill(const uint16_t *q, const uint16_t *k, const uint16_t *v,
                    const float *g, const float *beta, float *state, float *o,
                    int T, int Hk, int Hv, int D, float scale);

/* fp32 -> IEEE binary16 bits, round to nearest even (as __float2half_rn). */
uint16_t lio_fp32_to_fp16(float f);

/* Gated GQA attention layer, one decode step per sequence (the hybrid
 * stack's attention layers). Weights: w_in [2*Hq*D + 2*Hkv*D, hidden] with
 * rows q | gate | k | v; w_out [hidden, Hq*D]. KV caches are fp16 bits
 * [n_seqs][max_ctx][Hkv][D]; pos[s] is the slot of the new token (the number
 * of tokens already cached). Per sequence:
 *   p = W_in . rmsnorm?(x)
 *   q_h = rope(rmsnorm(q_h) * q_norm_w), k_j = rope(rmsnorm(k_j) * k_norm_w)
 *         (per-head RMSNorm skipped when the weight is NULL; NeoX rotate-half
 *         RoPE over the first rope_dim dims, angle pos * theta^(-2i/rope_dim))
 *   K[pos][j] = fp16(k_j), V[pos][j] = fp16(v_j)
 *   o_h = softmax_t(q_h . K[t][j] / sqrt(D)) V[t][j] over t = 0..pos,
 *         j = h / (Hq/Hkv), with the fp16 cache values
 *   y = W_out . (o * sigmoid(gate))
 * Double precision except the fp32 projection outputs and the fp16 cache. */
typedef struct lio_attn_layer {
    int hidden, n_q_heads, n_kv_heads, head_dim, rope_dim;
    int w_in_type, w_out_type;
    float rope_theta, in_norm_eps, qk_norm_eps;
    const float *in_norm_w;
    const void *w_in;
    const float *q_norm_w, *k_norm_w;
    const void *w_out;
} lio_attn_layer;

int lio_attn_layer_decode(const lio_attn_layer *L, const float *x, float *y,
                          uint16_t *k_cache, uint16_t *v_cache,
                          const int32_t *pos, int n_seqs, int max_ctx);

int lio_num_threads(void);

#ifdef __cplusplus
}
#endif
