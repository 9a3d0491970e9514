#pragma once

/*
 * LeanInfer fused-kernel C ABI, B200 (sm_100a) implementation.
 *
 * Drop-in for the reference header cuda/leaninfer-cuda.h: the five reference
 * entry points keep their exact names, argument lists and `void` returns, and
 * the header keeps the reference's dual shape (real declarations only when
 * GGML_USE_CUDA or GGML_USE_CUBLAS is defined, static no-op stubs otherwise;
 * reference cuda/leaninfer-cuda.h:16 and :54-76).
 *
 * Everything below the "additive entries" line is new. New entries return an
 * int status: 0 on success, a cudaError_t value for a CUDA failure, or one of
 * the LI_ERR_* codes for an argument the kernels do not accept.
 *
 * Conventions shared by all entries:
 *   - every pointer is device memory owned by the caller (ggml tensors);
 *     no entry allocates or frees device memory;
 *   - every launch is stream-ordered on `stream` (a cudaStream_t passed as
 *     void*, as in the reference) and performs no synchronisation and no
 *     host allocation; the entries that take their scratch from the caller
 *     may be captured into a CUDA graph;
 *   - quantized weights are raw ggml blocks, one matrix row after another
 *     (row r of a [N, K] matrix starts at r * li_row_bytes(type, K));
 *   - activations are fp32, row-major [n_rows, K].
 */

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml type ids, so a ggml dispatch can pass src0->type unchanged. */
enum li_wtype {
    LI_WTYPE_F32  = 0,
    LI_WTYPE_F16  = 1,
    LI_WTYPE_Q8_0 = 8,   /* 32 values per 34-byte block: fp16 d, 32 x int8   */
    LI_WTYPE_Q4_K = 12   /* 256 values per 144-byte block: fp16 d, fp16 dmin,
                            12 bytes of 6-bit scales/mins, 128 bytes of nibbles */
};

/* Status codes of the new entries (above every cudaError_t value). */
#define LI_OK                 0
#define LI_ERR_BAD_ARG        2001  /* null pointer, non-positive size      */
#define LI_ERR_BAD_SHAPE      2002  /* K not a multiple of the block size,
                                       or a size beyond what a kernel takes */
#define LI_ERR_UNSUPPORTED    2003  /* weight type / head_dim not built     */
#define LI_ERR_WORKSPACE      2004  /* workspace missing or too small       */
#define LI_ERR_MISALIGNED     2005  /* pointer not 16-byte aligned          */
#define LI_ERR_TIMEOUT        2006  /* a bounded device-side wait gave up   */
#define LI_ERR_NO_CUDA        2007  /* built without CUDA (stub branch)     */
#define LI_ERR_SCRATCH_LIMIT  2008  /* the call needs more scratch than the
                                       library's static scratch array holds */
#define LI_ERR_NCCL           2009  /* an NCCL call of a multi-GPU entry failed */

/* Size of the library's own device scratch used by
 * li_launch_deltanet_layer_decode_noalloc (32 MiB: every batch the tensor-core
 * decode path takes, up to 256 sequences, of a layer with hidden 4096,
 * 16 k-heads, 32 v-heads, head_dim 128). */
#define LI_DELTANET_STATIC_SCRATCH_BYTES (32u << 20)

/*
 * Recurrent DeltaNet layer for the fused decode entry. One layer's weights
 * and shapes; the per-sequence states live in caller buffers passed at launch.
 *
 * In-projection rows, in order (n_rows_in = 2*Hk*D + 2*Hv*D + 2*Hv):
 *   q [Hk*D] | k [Hk*D] | v [Hv*D] | z [Hv*D] | beta [Hv] | alpha [Hv]
 * Per step and sequence:
 *   p      = W_in . rmsnorm?(x)                (rmsnorm only if in_norm_w)
 *   c      = silu(causal_conv1d(p[q|k|v], conv_state, conv_w))  width 4
 *   q, k   = l2norm(c_q), l2norm(c_k) per k-head; q *= head_dim^-1/2
 *   beta   = sigmoid(p_beta)
 *   g      = -exp(a_log) * softplus(p_alpha + dt_bias)     (decay = e^g)
 *   S, o   = gated delta rule on S [D(k), D(v)] per v-head (see
 *            li_launch_deltanet_recurrent_f32)
 *   y      = W_out . ( silu(z) * rmsnorm(o) * norm_w )  per v-head rows
 */
typedef struct li_deltanet_layer {
    int   hidden;        /* model width K of W_in, rows of W_out        */
    int   n_k_heads;     /* Hk                                          */
    int   n_v_heads;     /* Hv, a multiple of Hk                        */
    int   head_dim;      /* D; 128 is the only built size               */
    int   conv_kernel;   /* 4 is the only built size                    */
    int   repeat_type;   /* 0: v-head h uses k-head h/(Hv/Hk);
                            1: v-head h uses k-head h % Hk               */
    int   w_in_type;     /* LI_WTYPE_Q4_K or LI_WTYPE_Q8_0              */
    int   w_out_type;    /* LI_WTYPE_Q4_K or LI_WTYPE_Q8_0              */
    float in_norm_eps;   /* eps of the optional input RMSNorm           */
    float norm_eps;      /* eps of the gated RMSNorm                    */
    float l2_eps;        /* eps of the q/k L2 normalisation             */
    const float *in_norm_w; /* [hidden] or NULL: no input RMSNorm       */
    const void  *w_in;      /* [n_rows_in, hidden] quantized rows        */
    const float *conv_w;    /* [2*Hk*D + Hv*D, conv_kernel]; tap
                               conv_kernel-1 multiplies the new input    */
    const float *a_log;     /* [Hv]                                      */
    const float *dt_bias;   /* [Hv]                                      */
    const float *norm_w;    /* [D] gamma of the gated RMSNorm            */
    const void  *w_out;     /* [hidden, Hv*D] quantized rows             */
} li_deltanet_layer;

/*
 * Gated GQA attention layer for the decode entry (the attention layers of the
 * hybrid DeltaNet / attention stack; the reference describes them in
 * docs/ASSESSMENT.md:1077 and :1086-1087 and has no kernel for them).
 *
 * In-projection rows, in order (n_rows_in = 2*Hq*D + 2*Hkv*D):
 *   q [Hq*D] | gate [Hq*D] | k [Hkv*D] | v [Hkv*D]
 * Per step and sequence s, the new token at position pos[s]:
 *   p      = W_in . rmsnorm?(x)                 (rmsnorm only if in_norm_w)
 *   q_h    = rope(rmsnorm(q_h) * q_norm_w)      per q head (norm skipped if NULL)
 *   k_j    = rope(rmsnorm(k_j) * k_norm_w)      per kv head
 *            rope: NeoX rotate-half over dims 0..rope_dim-1, angle of pair i
 *            pos * rope_theta^(-2i/rope_dim)
 *   K[s][pos][j] = f16(k_j), V[s][pos][j] = f16(v_j)
 *   o_h    = softmax_t(q_h . K[s][t][j] / sqrt(D)) V[s][t][j],  t = 0..pos,
 *            j = h / (Hq / Hkv)
 *   y      = W_out . (o * sigmoid(gate))
 */
typedef struct li_attn_layer {
    int   hidden;        /* model width K of W_in, rows of W_out          */
    int   n_q_heads;     /* Hq                                            */
    int   n_kv_heads;    /* Hkv; Hq / Hkv in 1..6 or 8                    */
    int   head_dim;      /* D; 128 is the only built size                 */
    int   rope_dim;      /* even, <= D; 0: no rotary embedding            */
    int   w_in_type;     /* LI_WTYPE_Q4_K or LI_WTYPE_Q8_0                */
    int   w_out_type;    /* LI_WTYPE_Q4_K or LI_WTYPE_Q8_0                */
    float rope_theta;    /* base of the rotary frequencies (> 1)          */
    float in_norm_eps;   /* eps of the optional input RMSNorm             */
    float qk_norm_eps;   /* eps of the per-head q / k RMSNorm             */
    const float *in_norm_w; /* [hidden] or NULL: no input RMSNorm         */
    const void  *w_in;      /* [n_rows_in, hidden] quantized rows          */
    const float *q_norm_w;  /* [D] or NULL                                 */
    const float *k_norm_w;  /* [D] or NULL                                 */
    const void  *w_out;     /* [hidden, Hq*D] quantized rows               */
} li_attn_layer;

/* One layer's SwiGLU FFN for the stack entry: y = W_down . (silu(W_gate . xn)
 * * (W_up . xn)), xn = rmsnorm(x) * norm_w. W_gate, W_up [n_inner, hidden];
 * W_down [hidden, n_inner]; with the weights sharded across GPUs, n_inner is
 * this rank's share and W_down holds the matching columns (see
 * li_launch_ffn_q_tp). */
typedef struct li_ffn_weights {
    int   wtype;         /* LI_WTYPE_Q4_K or LI_WTYPE_Q8_0                */
    int   hidden;
    int   n_inner;
    float eps;
    const float *norm_w;    /* [hidden] (NULL: no RMSNorm)                */
    const void  *w_gate;
    const void  *w_up;
    const void  *w_down;
} li_ffn_weights;

/* One layer of a hybrid decode stack: a mixer (DeltaNet or gated attention)
 * with its per-sequence state, followed by an FFN; both with residual adds. */
#define LI_LAYER_DELTANET 1
#define LI_LAYER_ATTN     2
typedef struct li_stack_layer {
    int kind;                            /* LI_LAYER_DELTANET or LI_LAYER_ATTN */
    const li_deltanet_layer *deltanet;   /* DELTANET: weights (in_norm_w is the pre-norm) */
    float *conv_state;                   /* DELTANET: [n_seqs][C][3]               */
    float *state;                        /* DELTANET: [n_seqs][Hv][D][D]           */
    const li_attn_layer *attn;           /* ATTN: weights (in_norm_w is the pre-norm) */
    void  *k_cache, *v_cache;            /* ATTN: __half [n_seqs][max_ctx][Hkv][D] */
    li_ffn_weights ffn;
} li_stack_layer;

#if defined(GGML_USE_CUDA) || defined(GGML_USE_CUBLAS)

/* ======================================================================
 * Reference entries (reference cuda/leaninfer-cuda.h:19-52), unchanged
 * signatures. Errors are recorded for li_get_last_error().
 * ====================================================================== */

/* dst[r][n] = sum_k rmsnorm(x[r])[k] * W[n][k], fp32 W [N, K].
 * Replaces reference cuda/leaninfer-fused-ffn.cu:259-268 (one row of x). */
void li_launch_fused_rms_norm_matmul_f32(
        const float * x, const float * gamma, const float * W,
        float * dst, int K, int N, float eps, void * stream);

/* hidden[n] = silu(<x_norm, W_gate[n]>) * <x_norm, W_up[n]>, fp32 weights.
 * Replaces reference cuda/leaninfer-fused-ffn.cu:270-280. */
void li_launch_fused_rms_norm_swiglu_f32(
        const float * x, const float * gamma,
        const float * W_gate, const float * W_up,
        float * hidden, int K, int N, float eps, void * stream);

/* Same with fp16 weights (const void* = half[N*K]); x_norm is rounded to
 * fp16 before the dot, as in reference cuda/leaninfer-fused-ffn.cu:230.
 * Replaces reference cuda/leaninfer-fused-ffn.cu:282-292. */
void li_launch_fused_rms_norm_swiglu_f16(
        const float * x, const float * gamma,
        const void  * W_gate, const void  * W_up,
        float * hidden, int K, int N, float eps, void * stream);

/* dst[r][k] = silu(z[r][k]) * output[r][k] * gamma[k] * rsqrt(mean(output[r]^2)+eps).
 * Replaces reference cuda/leaninfer-fused-gate.cu:92-99. */
void li_launch_fused_rms_norm_silu_gate_f32(
        const float * output, const float * z, const float * gamma,
        float * dst, int K, int n_rows, float eps, void * stream);

/* Gated delta-rule recurrence over n_tokens with the reference layouts
 * (reference cuda/leaninfer-fused-deltanet.cu:331-366):
 *   q, k  [n_seqs][n_heads/gqa][n_tokens][D]; v addressed with element
 *   strides vnb1 (token), vnb2 (head), vnb3 (seq); g, beta [n_seqs][n_tokens][n_heads];
 *   state_in [n_seqs][n_heads][D(k)][D(v)];
 *   dst = per-head outputs [n_seqs][n_tokens][n_heads][D], followed by the
 *   final state in the state_in layout.
 * proj_out [hidden_dim][n_tokens] receives sum over seqs and heads of
 * W_out[d][h*D + j] * o[h][j] (W_out fp32 [hidden_dim, n_heads*D]); it is
 * zeroed first. head_dim 128 and 64 are built; any other value records
 * LI_ERR_UNSUPPORTED. */
void li_launch_fused_deltanet_recurrent_out_f32(
        const float * q, const float * k, const float * v,
        const float * g, const float * beta, const float * state_in,
        const float * W_out,
        float * dst, float * proj_out,
        int64_t head_dim, int64_t n_tokens, int64_t n_heads,
        int64_t gqa_ratio, int repeat_type, int64_t n_seqs,
        int64_t hidden_dim,
        size_t vnb1, size_t vnb2, size_t vnb3,
        void * stream);

/* RMSNorm + three fp32 projections sharing one normalised x:
 * dst_ptrs[i][n] = <rmsnorm(x), W_ptrs[i][n]>, i = 0..2, each W [N_OUT, K].
 * W_ptrs and dst_ptrs are arrays of three device pointers, both in device
 * memory (as the reference's comment asks, "pass device-side pointer
 * arrays"; the kernel reads them when it runs, so a captured graph follows
 * later changes to the arrays) or both in host memory (read at launch).
 * The side is found with cudaPointerGetAttributes; arrays on different sides
 * record LI_ERR_BAD_ARG. The reference exports this symbol as a stub
 * (reference cuda/leaninfer-fused-deltanet.cu:306-327). */
void li_launch_fused_rms_norm_qkv_f32(
        const float * x, const float * gamma,
        const float * const * W_ptrs,
        float * const * dst_ptrs,
        int K, int N_OUT, float eps, void * stream);

/* Status of the last reference-entry launch on the calling host thread
 * (0 = success). Reading it clears it. */
int li_get_last_error(void);

/* ======================================================================
 * Additive entries (no reference counterpart unless cited).
 * ====================================================================== */

/* Synchronises the current device and returns (and clears) the status of
 * the bounded device-side waits of earlier launches: LI_ERR_TIMEOUT if one
 * gave up, a cudaError_t value if the synchronisation failed, else 0.
 * Synchronous: not for use inside graph capture. */
int li_device_status(void);

/* Bytes of one row of k values of type wtype (0 if k is not a multiple of
 * the block size or the type is unknown). */
size_t li_row_bytes(int wtype, int64_t k);

/* Diagnostic of the bounded device-side waits (no counterpart in the
 * reference, which has no device-side failure reporting). Launches one small
 * kernel whose mbarrier wait can never complete, with the library's bounded
 * wait cut to limit_us microseconds (1 .. 1000000): the wait gives up, the
 * kernel returns by itself, and the next li_device_status() reports
 * LI_ERR_TIMEOUT, exactly as when a wait of a real kernel runs out. If
 * elapsed_ns is not NULL (device memory), the kernel stores how long the wait
 * ran before giving up. Returns the launch status. */
int li_selftest_bounded_wait(int limit_us, unsigned long long * elapsed_ns, void * stream);

/* dst[i] = a[i] + b[i], i < n (fp32; dst may alias a or b): the residual
 * connection between the layers of a decode stack (ggml ADD). */
int li_launch_add_f32(float * dst, const float * a, const float * b, int64_t n, void * stream);

/* Block decode to fp32 (ggml to_float, as called from reference
 * metal/leaninfer-metal.mm:187-193). Bit-exact with gguf-py's dequantize for
 * Q8_0 and Q4_K. n = number of values (a multiple of the block size). */
int li_launch_dequantize(int wtype, const void * src, float * dst, int64_t n,
                         void * stream);

/* dst[r][n] = <rmsnorm(x[r]) or x[r], W[n]> over n_rows rows of x.
 * gamma == NULL skips the RMSNorm (plain quantized matmul, e.g. the FFN
 * down projection). Quantized counterpart of
 * reference cuda/leaninfer-fused-ffn.cu:41-97. */
int li_launch_rms_norm_matmul_q(int wtype,
        const float * x, const float * gamma, const void * W, float * dst,
        int K, int N, int n_rows, float eps, void * stream);

/* RMSNorm + Q/K/V projections with one shared normalised x (the reference's
 * intended li_fused_rms_norm_multi_proj_f32<3>,
 * reference cuda/leaninfer-fused-deltanet.cu:46-110). */
int li_launch_fused_rms_norm_qkv_q(int wtype,
        const float * x, const float * gamma,
        const void * Wq, const void * Wk, const void * Wv,
        float * q, float * k, float * v,
        int K, int Nq, int Nk, int Nv, int n_rows, float eps, void * stream);

/* RMSNorm + SwiGLU gate/up (quantized counterpart of
 * reference cuda/leaninfer-fused-ffn.cu:116-180):
 * h[r][n] = silu(<x_norm, Wg[n]>) * <x_norm, Wu[n]>. */
int li_launch_fused_rms_norm_swiglu_q(int wtype,
        const float * x, const float * gamma,
        const void * Wg, const void * Wu, float * h,
        int K, int N, int n_rows, float eps, void * stream);

/* Whole SwiGLU FFN: y = Wd . (silu(Wg.xn) * (Wu.xn)), xn = rmsnorm(x).
 * Wg, Wu [N, K]; Wd [K, N]. The intermediate h (and, from 3 rows on, the
 * f16 operands of the tensor-core path) live in the workspace. */
size_t li_fused_ffn_workspace_size(int K, int N, int n_rows);
int li_launch_fused_ffn_q(int wtype,
        const float * x, const float * gamma,
        const void * Wg, const void * Wu, const void * Wd, float * y,
        int K, int N, int n_rows, float eps,
        void * workspace, size_t workspace_bytes, void * stream);

/* Gated delta-rule recurrence with the reference's arithmetic and layouts
 * (same argument meaning as li_launch_fused_deltanet_recurrent_out_f32,
 * without the projection): writes per-head outputs to `out`
 * [n_seqs][n_tokens][n_heads][D] and the final state to state_out
 * (state_out == state_in is allowed: each head's state is read fully before
 * it is written, by the same thread block). Recurrence per token
 * (reference cuda/leaninfer-fused-deltanet.cu:217-288):
 *   q~ = q * D^-1/2, beta = sigmoid(beta_in), a = exp(min(g, 50)),
 *   u = S^T k, w = S^T q~, v' = beta (v - a u), o = a w + v' (k . q~),
 *   S <- clamp(a S + k v'^T, -1e6, 1e6). */
int li_launch_deltanet_recurrent_f32(
        const float * q, const float * k, const float * v,
        const float * g, const float * beta, const float * state_in,
        float * out, float * state_out,
        int64_t head_dim, int64_t n_tokens, int64_t n_heads,
        int64_t gqa_ratio, int repeat_type, int64_t n_seqs,
        size_t vnb1, size_t vnb2, size_t vnb3, void * stream);

/* One decode step (one token per sequence) of a whole DeltaNet layer, as
 * described at li_deltanet_layer. x, y [n_seqs, hidden]; conv_state
 * [n_seqs][2*Hk*D + Hv*D][conv_kernel-1] (oldest input first) and
 * state [n_seqs][Hv][D(k)][D(v)] are updated in place. */
size_t li_deltanet_layer_workspace_size(const li_deltanet_layer * L, int n_seqs);
int li_launch_deltanet_layer_decode(const li_deltanet_layer * L,
        const float * x, float * y, float * conv_state, float * state,
        int n_seqs, void * workspace, size_t workspace_bytes, void * stream);

/* The same step with the recurrent state stored as fp16 (`state` is
 * __half [n_seqs][Hv][D][D], the fp32 entry's element order), computed in
 * fp32 and rounded once per step when stored, saturating at +-65504 (the
 * reference's +-1e6 clamp lies beyond the fp16 range). Half the state bytes
 * of the fp32 entry. No counterpart among the reference's kernels: upstream's
 * fp16 recurrent-state storage option (reference docs/RESULTS.md:37). Same
 * workspace size. */
int li_launch_deltanet_layer_decode_f16state(const li_deltanet_layer * L,
        const float * x, float * y, float * conv_state, void * state,
        int n_seqs, void * workspace, size_t workspace_bytes, void * stream);

/* The same layer decode step for callers that cannot allocate device memory
 * for a workspace (for example a ggml graph whose buffers were all planned
 * before this op, or a host runtime that owns every device allocation and
 * passes only tensors and a stream). This entry has no counterpart in the
 * reference. Its scratch is a device array inside the library
 * (LI_DELTANET_STATIC_SCRATCH_BYTES, held by every GPU that loads the
 * library until the process exits); the call allocates nothing. A call whose
 * workspace would exceed it returns LI_ERR_SCRATCH_LIMIT without launching.
 * The first call on a device looks up the array's device address (with that
 * device current), so make that first call before any stream capture. All
 * calls share the one array: calls that overlap on the GPU (for example on
 * two streams at once) race on it and must be serialised by the caller.
 * Nothing in the scratch needs to start at zero. */
int li_launch_deltanet_layer_decode_noalloc(const li_deltanet_layer * L,
        const float * x, float * y, float * conv_state, float * state,
        int n_seqs, void * stream);

/* One decode step (one token per sequence) of the gated attention layer
 * described at li_attn_layer. x, y [n_seqs, hidden] fp32; k_cache and
 * v_cache are __half [n_seqs][max_ctx][Hkv][D] (token-major, as ggml's KV
 * cache rows); pos [n_seqs] int32 in device memory, 0 <= pos[s] < max_ctx:
 * the step writes the new token's k and v at pos[s] and attends over tokens
 * 0..pos[s]; the caller advances pos between steps. A position outside
 * [0, max_ctx) (the host cannot see device memory to check it) writes and
 * reads no cache row: that sequence's output is the out-projection of zeros
 * and li_device_status() reports LI_ERR_BAD_ARG. No counterpart among the
 * reference's kernels. */
size_t li_attn_layer_workspace_size(const li_attn_layer * L, int n_seqs, int max_ctx);
int li_launch_attn_layer_decode(const li_attn_layer * L,
        const float * x, float * y, void * k_cache, void * v_cache,
        const int32_t * pos, int n_seqs, int max_ctx,
        void * workspace, size_t workspace_bytes, void * stream);

/* ----------------------------------------------------------------------
 * Multi-GPU: the SwiGLU FFN sharded two ways over NCCL (no counterpart in
 * the reference, which has no multi-GPU code). Sequences stay sharded by rank
 * (rows_per_rank rows of x and y per rank, the same count on every rank);
 * the FFN's inner dimension is split into block-aligned ranges, one per rank:
 * this rank holds W_gate and W_up rows [n0, n0 + N_local) and the matching
 * byte range of every W_down row (W_down shard [K, N_local], row stride
 * li_row_bytes(wtype, N_local)). A step all-gathers x over the communicator,
 * runs li_launch_fused_ffn_q on all nranks * rows_per_rank rows with the
 * local shard, and reduce-scatters (sums) the partial outputs back to this
 * rank's rows of y. `comm` is an ncclComm_t of nranks ranks (one per GPU);
 * NCCL is loaded with dlopen("libnccl.so.2") at first use, the copy already
 * in the process when there is one. Every rank calls with the same shapes in
 * the same order. Returns LI_ERR_NCCL if an NCCL call fails,
 * LI_ERR_UNSUPPORTED if no NCCL library can be loaded. With nranks == 1 it
 * is li_launch_fused_ffn_q (comm unused).
 * ---------------------------------------------------------------------- */
int li_nccl_available(void);
int li_nccl_get_unique_id(void * id);   /* 128 bytes (ncclUniqueId) */
int li_nccl_comm_init_rank(void ** comm, int nranks, const void * id, int rank);
int li_nccl_comm_destroy(void * comm);
size_t li_ffn_tp_workspace_size(int K, int N_local, int rows_per_rank, int nranks);
int li_launch_ffn_q_tp(int wtype,
        const float * x, const float * gamma,
        const void * Wg, const void * Wu, const void * Wd, float * y,
        int K, int N_local, int rows_per_rank, float eps,
        void * comm, int nranks,
        void * workspace, size_t workspace_bytes, void * stream);

/* One decode step of a hybrid layer stack for n_seqs sequences (one token
 * each): for every layer in order, x += mixer(x), then x += ffn(x), where x
 * [n_seqs][hidden] fp32 is the residual stream, updated in place; the mixers
 * update their states and caches in place (attention layers write slot
 * pos[s]). With tp_nranks > 1 every FFN runs as li_launch_ffn_q_tp over
 * tp_comm (an ncclComm_t) with this rank's FFN shards. No counterpart in the
 * reference: the composition of the reference product's decode graph
 * (docs/ASSESSMENT.md:1073-1090) over this library's layer entries. */
size_t li_stack_workspace_size(const li_stack_layer * layers, int n_layers, int n_seqs, int max_ctx,
        int tp_nranks);
int li_launch_stack_decode(const li_stack_layer * layers, int n_layers, float * x,
        const int32_t * pos, int n_seqs, int max_ctx, void * tp_comm, int tp_nranks,
        void * workspace, size_t workspace_bytes, void * stream);

/* Chunked (WY form, chunk 64) gated delta rule prefill of one sequence of T
 * tokens on the tensor cores (bf16 operands, fp32 accumulation and state).
 * No counterpart in the reference (its prefill is the upstream per-token
 * DELTA_NET op); the arithmetic is the token recurrence
 *   a = exp(g), q~ = scale q, v' = beta (v - a S^T k), S <- a S + k v'^T,
 *   o = S^T q~
 * (beta already a gate in (0,1), no clamp). Layouts: q, k bf16
 * [T][n_k_heads][head_dim]; v bf16 [T][n_v_heads][head_dim]; g (log decay),
 * beta fp32 [T][n_v_heads]; state fp32 [n_v_heads][D(k)][D(v)], updated in
 * place to the state after token T-1; o fp32 [T][n_v_heads][head_dim]. v-head
 * h reads k-head h / (n_v_heads / n_k_heads). head_dim 128. q, k, v and the
 * workspace 16-byte aligned. */
size_t li_deltanet_chunk_prefill_workspace_size(int T, int n_v_heads, int head_dim);
int li_launch_deltanet_chunk_prefill_bf16(const void * q, const void * k, const void * v,
        const float * g, const float * beta, float * state, float * o,
        int T, int n_k_heads, int n_v_heads, int head_dim, float scale,
        void * workspace, size_t workspace_bytes, void * stream);

/* The prefill's output stage (no counterpart in the reference). Gated RMSNorm
 * of n_rows rows of K values written as bf16:
 *   dst = bf16(silu(z) * (o * gamma * rsqrt(mean(o^2) + eps)))
 * (the arithmetic of li_launch_fused_rms_norm_silu_gate_f32); and a bf16
 * GEMM on the tensor cores, C[M][N] (fp32, row-major) = A[M][K] . W[N][K]^T
 * with A and W bf16 row-major (fp32 accumulation); M a multiple of 128, N of
 * 256, K of 64; A, W, C 16-byte aligned. The norm needs K % 4 == 0, o, z,
 * gamma 16-byte and dst 8-byte aligned. */
int li_launch_gated_rmsnorm_bf16(const float * o, const float * z, const float * gamma,
        void * dst, int K, int64_t n_rows, float eps, void * stream);
int li_launch_gemm_bf16_f32(const void * A, const void * W, float * C,
        int M, int N, int K, void * stream);

#else  /* no CUDA: the reference's no-op stubs, plus stubs for the new entries */

static inline void li_launch_fused_rms_norm_silu_gate_f32(
        const float*o,const float*z,const float*g,float*d,int K,int nr,float e,void*s)
        {(void)o;(void)z;(void)g;(void)d;(void)K;(void)nr;(void)e;(void)s;}
static inline void li_launch_fused_rms_norm_matmul_f32(
        const float*x,const float*g,const float*W,float*d,int K,int N,float e,void*s)
        {(void)x;(void)g;(void)W;(void)d;(void)K;(void)N;(void)e;(void)s;}
static inline void li_launch_fused_rms_norm_swiglu_f32(
        const float*x,const float*g,const float*wg,const float*wu,float*h,int K,int N,float e,void*s)
        {(void)x;(void)g;(void)wg;(void)wu;(void)h;(void)K;(void)N;(void)e;(void)s;}
static inline void li_launch_fused_rms_norm_swiglu_f16(
        const float*x,const float*g,const void*wg,const void*wu,float*h,int K,int N,float e,void*s)
        {(void)x;(void)g;(void)wg;(void)wu;(void)h;(void)K;(void)N;(void)e;(void)s;}
static inline void li_launch_fused_deltanet_recurrent_out_f32(
        const float*q,const float*k,const float*v,const float*g,const float*b,const float*s,
        const float*w,float*d,float*p,int64_t hd,int64_t nt,int64_t nh,int64_t gr,int rt,
        int64_t ns,int64_t hid,size_t v1,size_t v2,size_t v3,void*st)
        {(void)q;(void)k;(void)v;(void)g;(void)b;(void)s;(void)w;(void)d;(void)p;
         (void)hd;(void)nt;(void)nh;(void)gr;(void)rt;(void)ns;(void)hid;(void)v1;(void)v2;(void)v3;(void)st;}
static inline void li_launch_fused_rms_norm_qkv_f32(
        const float*x,const float*g,const float*const*W,float*const*d,int K,int N,float e,void*s)
        {(void)x;(void)g;(void)W;(void)d;(void)K;(void)N;(void)e;(void)s;}
static inline int li_get_last_error(void) { return LI_ERR_NO_CUDA; }

/* The additive entries without CUDA: each returns LI_ERR_NO_CUDA (sizes 0),
 * so a caller compiled without GGML_USE_CUDA still compiles and links. The
 * row size is host arithmetic and keeps its meaning. */
static inline int li_device_status(void) { return LI_ERR_NO_CUDA; }
static inline int li_selftest_bounded_wait(int l, unsigned long long*e, void*s)
        {(void)l;(void)e;(void)s; return LI_ERR_NO_CUDA;}
static inline size_t li_row_bytes(int t, int64_t k) {
    if (k <= 0) return 0;
    if (t == LI_WTYPE_F32) return (size_t)k * 4;
    if (t == LI_WTYPE_F16) return (size_t)k * 2;
    if (t == LI_WTYPE_Q8_0) return (k % 32) ? 0 : (size_t)(k / 32) * 34;
    if (t == LI_WTYPE_Q4_K) return (k % 256) ? 0 : (size_t)(k / 256) * 144;
    return 0;
}
static inline int li_launch_add_f32(float*d, const float*a, const float*b, int64_t n, void*s)
        {(void)d;(void)a;(void)b;(void)n;(void)s; return LI_ERR_NO_CUDA;}
static inline int li_launch_dequantize(int t, const void*s, float*d, int64_t n, void*st)
        {(void)t;(void)s;(void)d;(void)n;(void)st; return LI_ERR_NO_CUDA;}
static inline int li_launch_rms_norm_matmul_q(int t, const float*x, const float*g, const void*W, float*d,
        int K, int N, int r, float e, void*s)
        {(void)t;(void)x;(void)g;(void)W;(void)d;(void)K;(void)N;(void)r;(void)e;(void)s; return LI_ERR_NO_CUDA;}
static inline int li_launch_fused_rms_norm_qkv_q(int t, const float*x, const float*g,
        const void*wq, const void*wk, const void*wv, float*q, float*k, float*v,
        int K, int nq, int nk, int nv, int r, float e, void*s)
        {(void)t;(void)x;(void)g;(void)wq;(void)wk;(void)wv;(void)q;(void)k;(void)v;(void)K;(void)nq;(void)nk;
         (void)nv;(void)r;(void)e;(void)s; return LI_ERR_NO_CUDA;}
static inline int li_launch_fused_rms_norm_swiglu_q(int t, const float*x, const float*g,
        const void*wg, const void*wu, float*h, int K, int N, int r, float e, void*s)
        {(void)t;(void)x;(void)g;(void)wg;(void)wu;(void)h;(void)K;(void)N;(void)r;(void)e;(void)s;
         return LI_ERR_NO_CUDA;}
static inline size_t li_fused_ffn_workspace_size(int K, int N, int r) {(void)K;(void)N;(void)r; return 0;}
static inline int li_launch_fused_ffn_q(int t, const float*x, const float*g,
        const void*wg, const void*wu, const void*wd, float*y, int K, int N, int r, float e,
        void*ws, size_t wb, void*s)
        {(void)t;(void)x;(void)g;(void)wg;(void)wu;(void)wd;(void)y;(void)K;(void)N;(void)r;(void)e;(void)ws;
         (void)wb;(void)s; return LI_ERR_NO_CUDA;}
static inline int li_launch_deltanet_recurrent_f32(const float*q, const float*k, const float*v,
        const float*g, const float*b, const float*si, float*o, float*so,
        int64_t hd, int64_t nt, int64_t nh, int64_t gr, int rt, int64_t ns,
        size_t v1, size_t v2, size_t v3, void*s)
        {(void)q;(void)k;(void)v;(void)g;(void)b;(void)si;(void)o;(void)so;(void)hd;(void)nt;(void)nh;(void)gr;
         (void)rt;(void)ns;(void)v1;(void)v2;(void)v3;(void)s; return LI_ERR_NO_CUDA;}
static inline size_t li_deltanet_layer_workspace_size(const li_deltanet_layer*L, int n)
        {(void)L;(void)n; return 0;}
static inline int li_launch_deltanet_layer_decode(const li_deltanet_layer*L, const float*x, float*y,
        float*cs, float*st, int n, void*ws, size_t wb, void*s)
        {(void)L;(void)x;(void)y;(void)cs;(void)st;(void)n;(void)ws;(void)wb;(void)s; return LI_ERR_NO_CUDA;}
static inline int li_launch_deltanet_layer_decode_f16state(const li_deltanet_layer*L, const float*x, float*y,
        float*cs, void*st, int n, void*ws, size_t wb, void*s)
        {(void)L;(void)x;(void)y;(void)cs;(void)st;(void)n;(void)ws;(void)wb;(void)s; return LI_ERR_NO_CUDA;}
static inline int li_launch_deltanet_layer_decode_noalloc(const li_deltanet_layer*L, const float*x, float*y,
        float*cs, float*st, int n, void*s)
        {(void)L;(void)x;(void)y;(void)cs;(void)st;(void)n;(void)s; return LI_ERR_NO_CUDA;}
static inline size_t li_attn_layer_workspace_size(const li_attn_layer*L, int n, int c)
        {(void)L;(void)n;(void)c; return 0;}
static inline int li_launch_attn_layer_decode(const li_attn_layer*L, const float*x, float*y, void*kc, void*vc,
        const int32_t*p, int n, int c, void*ws, size_t wb, void*s)
        {(void)L;(void)x;(void)y;(void)kc;(void)vc;(void)p;(void)n;(void)c;(void)ws;(void)wb;(void)s;
         return LI_ERR_NO_CUDA;}
static inline int li_nccl_available(void) { return 0; }
static inline int li_nccl_get_unique_id(void*id) {(void)id; return LI_ERR_NO_CUDA;}
static inline int li_nccl_comm_init_rank(void**c, int n, const void*id, int r)
        {(void)c;(void)n;(void)id;(void)r; return LI_ERR_NO_CUDA;}
static inline int li_nccl_comm_destroy(void*c) {(void)c; return LI_ERR_NO_CUDA;}
static inline size_t li_ffn_tp_workspace_size(int K, int N, int r, int n) {(void)K;(void)N;(void)r;(void)n; return 0;}
static inline int li_launch_ffn_q_tp(int t, const float*x, const float*g, const void*wg, const void*wu,
        const void*wd, float*y, int K, int N, int r, float e, void*c, int n, void*ws, size_t wb, void*s)
        {(void)t;(void)x;(void)g;(void)wg;(void)wu;(void)wd;(void)y;(void)K;(void)N;(void)r;(void)e;(void)c;(void)n;
         (void)ws;(void)wb;(void)s; return LI_ERR_NO_CUDA;}
static inline size_t li_stack_workspace_size(const li_stack_layer*l, int nl, int n, int c, int tp)
        {(void)l;(void)nl;(void)n;(void)c;(void)tp; return 0;}
static inline int li_launch_stack_decode(const li_stack_layer*l, int nl, float*x, const int32_t*p, int n, int c,
        void*comm, int tp, void*ws, size_t wb, void*s)
        {(void)l;(void)nl;(void)x;(void)p;(void)n;(void)c;(void)comm;(void)tp;(void)ws;(void)wb;(void)s;
         return LI_ERR_NO_CUDA;}
static inline size_t li_deltanet_chunk_prefill_workspace_size(int T, int hv, int hd)
        {(void)T;(void)hv;(void)hd; return 0;}
static inline int li_launch_deltanet_chunk_prefill_bf16(const void*q, const void*k, const void*v,
        const float*g, const float*b, float*st, float*o, int T, int hk, int hv, int hd, float sc,
        void*ws, size_t wb, void*s)
        {(void)q;(void)k;(void)v;(void)g;(void)b;(void)st;(void)o;(void)T;(void)hk;(void)hv;(void)hd;(void)sc;
         (void)ws;(void)wb;(void)s; return LI_ERR_NO_CUDA;}
static inline int li_launch_gated_rmsnorm_bf16(const float*o, const float*z, const float*g, void*d, int K,
        int64_t n, float e, void*s)
        {(void)o;(void)z;(void)g;(void)d;(void)K;(void)n;(void)e;(void)s; return LI_ERR_NO_CUDA;}
static inline int li_launch_gemm_bf16_f32(const void*A, const void*W, float*C, int M, int N, int K, void*s)
        {(void)A;(void)W;(void)C;(void)M;(void)N;(void)K;(void)s; return LI_ERR_NO_CUDA;}

#endif

#ifdef __cplusplus
}
#endif
