/*
 * ggml-style dispatch onto the LeanInfer B200 entries (host C API).
 *
 * The reference plugs its ops into ggml-cuda as new GGML_OP_* cases of
 * ggml_cuda_compute_forward that read the node's sources, shapes and op
 * parameters and launch on ctx.stream() (reference
 * scripts/patch_fused_gate.sh:167-204). li_ggml_compute_forward is that
 * dispatch as one testable function: it reads a node described by
 * li_ggml_tensor (the fields of ggml_tensor the dispatch uses, with ggml's
 * meaning: ne[0] is the contiguous dimension, nb[i] the byte stride of
 * dimension i, src[] the operands, op_params the op's parameters), checks
 * types, shapes and strides as ggml's supports_op would, and calls the
 * matching entry of leaninfer-cuda.h on the caller's stream. A ggml-cuda
 * case fills the descriptor from its ggml_tensor field by field.
 *
 * Nodes (M = rows of the activation, i.e. ne[1] * ne[2] * ne[3]):
 *   LI_GGML_OP_MUL_MAT          dst f32 [N, M] = src1 . src0^T with src0
 *                               Q8_0 / Q4_K [K, N] and src1 f32 [K, M]
 *                               (ggml MUL_MAT) -> li_launch_rms_norm_matmul_q
 *                               without the norm.
 *   LI_GGML_OP_FUSED_UP_GATE    dst f32 [N, M] = silu(x . W_gate^T) *
 *                               (x . W_up^T), src0 = W_up, src1 = W_gate
 *                               (Q8_0 / Q4_K [K, N]), src2 = x f32 [K, M],
 *                               already normalised (reference
 *                               metal/leaninfer-metal.mm:239-243)
 *                               -> li_launch_fused_rms_norm_swiglu_q.
 *   LI_GGML_OP_FUSED_RMS_SILU_GATE  dst = silu(z) * (o * gamma *
 *                               rsqrt(mean(o^2) + eps)) per row of K =
 *                               src0->ne[0]; src0 = o, src1 = z (f32, same
 *                               shape), src2 = gamma f32 [K], eps =
 *                               op_params[0] as a float (reference
 *                               scripts/patch_fused_gate.sh:167-178)
 *                               -> li_launch_fused_rms_norm_silu_gate_f32.
 *   LI_GGML_OP_DELTANET_DECODE  one decode step of a Gated DeltaNet layer
 *                               for n_seqs sequences -> li_launch_deltanet_
 *                               layer_decode; dst = y f32 [hidden, n_seqs];
 *                               src0 x f32 [hidden, n_seqs];
 *                               src1 conv state f32 [3, C, n_seqs] (C = 2 Hk D
 *                               + Hv D), updated in place;
 *                               src2 recurrent state f32 or f16 [D, D, Hv,
 *                               n_seqs] ([seq][v-head][k][v]), updated in
 *                               place (f16: li_launch_deltanet_layer_decode_
 *                               f16state);
 *                               src3 W_in Q8_0 / Q4_K [hidden, 2 Hk D + 2 Hv D
 *                               + 2 Hv]; src4 conv weights f32 [4, C];
 *                               src5 a_log f32 [Hv]; src6 dt_bias f32 [Hv];
 *                               src7 gated-norm gamma f32 [D]; src8 W_out
 *                               Q8_0 / Q4_K [Hv D, hidden]; src9 input-norm
 *                               gamma f32 [hidden] or NULL;
 *                               op_params[0] = Hk, [1] = repeat_type,
 *                               [2] / [3] / [4] = l2 / gated-norm / input-norm
 *                               eps as floats. Needs a workspace of
 *                               li_ggml_workspace_size(node) bytes.
 *
 * Every tensor must be contiguous (f32: nb[0] = 4 and nb[i+1] = nb[i] *
 * ne[i]; quantized: nb[1] = the row size of ne[0] values, higher strides
 * contiguous over rows). Returns LI_OK, LI_ERR_BAD_ARG (null node, source or
 * data), LI_ERR_UNSUPPORTED (op or type), LI_ERR_BAD_SHAPE (shapes that do
 * not match, or strides that are not contiguous), or the entry's own status.
 */
#ifndef LEANINFER_GGML_H
#define LEANINFER_GGML_H

#include <stddef.h>
#include <stdint.h>

#include "leaninfer-cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

enum li_ggml_type {
    LI_GGML_TYPE_F32  = 0,
    LI_GGML_TYPE_F16  = 1,
    LI_GGML_TYPE_Q8_0 = 8,
    LI_GGML_TYPE_Q4_K = 12
};

enum li_ggml_op {
    LI_GGML_OP_NONE = 0,
    LI_GGML_OP_MUL_MAT = 1,
    LI_GGML_OP_FUSED_UP_GATE = 2,
    LI_GGML_OP_FUSED_RMS_SILU_GATE = 3,
    LI_GGML_OP_DELTANET_DECODE = 4
};

#define LI_GGML_MAX_DIMS 4
#define LI_GGML_MAX_SRC 10
#define LI_GGML_MAX_OP_PARAMS 16   /* int32 words (ggml: 64 bytes) */

typedef struct li_ggml_tensor {
    int32_t type;                               /* enum li_ggml_type */
    int64_t ne[LI_GGML_MAX_DIMS];               /* elements per dimension */
    size_t  nb[LI_GGML_MAX_DIMS];               /* byte stride per dimension */
    int32_t op;                                 /* enum li_ggml_op (nodes) */
    int32_t op_params[LI_GGML_MAX_OP_PARAMS];
    struct li_ggml_tensor *src[LI_GGML_MAX_SRC];
    void   *data;                               /* device memory */
} li_ggml_tensor;

#if defined(GGML_USE_CUDA) || defined(GGML_USE_CUBLAS)

/* Workspace bytes the node needs (0 for all but LI_GGML_OP_DELTANET_DECODE). */
size_t li_ggml_workspace_size(const li_ggml_tensor *node);

/* Runs the node on `stream` (a cudaStream_t); capture-safe like the entries. */
int li_ggml_compute_forward(const li_ggml_tensor *node, void *workspace, size_t workspace_bytes,
                            void *stream);

#else  /* no CUDA: the same dual shape as leaninfer-cuda.h */

static inline size_t li_ggml_workspace_size(const li_ggml_tensor *node) { (void)node; return 0; }
static inline int li_ggml_compute_forward(const li_ggml_tensor *node, void *workspace, size_t workspace_bytes,
                                          void *stream)
        {(void)node;(void)workspace;(void)workspace_bytes;(void)stream; return LI_ERR_NO_CUDA;}

#endif

#ifdef __cplusplus
}
#endif

#endif /* LEANINFER_GGML_H */
