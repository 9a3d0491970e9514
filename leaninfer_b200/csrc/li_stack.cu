// Decode step of a hybrid Gated DeltaNet / gated-attention layer stack (the
// Qwen3.5-style stack the reference describes in docs/ASSESSMENT.md:1073-1090:
// repeating blocks of DeltaNet + FFN and attention + FFN layers).
//
// The residual stream x [n_seqs][hidden] (fp32) is updated in place, layer by
// layer:
//     x += mixer(x)          li_launch_deltanet_layer_decode (its input RMSNorm
//                            weight is the layer's pre-norm) or
//                            li_launch_attn_layer_decode
//     x += ffn(x)            li_launch_fused_ffn_q (RMSNorm + SwiGLU + down),
//                            or li_launch_ffn_q_tp over a communicator when the
//                            FFN weights are sharded across GPUs
// The mixers and the unsharded FFN run in their residual forms: their output
// projection adds its result into x, so no residual-add kernel runs between
// them (the sharded FFN's result is added by li_launch_add_f32).
// Every launch goes to the caller's stream; the host loop only issues them
// (nothing synchronises), so a whole step can be captured into one CUDA graph.
// Embeddings and the output head are not part of the stack.
#include "li_common.cuh"

namespace li {
namespace {

size_t al256(size_t v) { return (v + 255) / 256 * 256; }

size_t ffn_ws(const li_stack_layer &l, int n, int tp) {
    return tp > 1 ? li_ffn_tp_workspace_size(l.ffn.hidden, l.ffn.n_inner, n, tp)
                  : li_fused_ffn_workspace_size(l.ffn.hidden, l.ffn.n_inner, n);
}

size_t mixer_ws(const li_stack_layer &l, int n, int max_ctx) {
    if (l.kind == LI_LAYER_DELTANET) return li_deltanet_layer_workspace_size(l.deltanet, n);
    return li_attn_layer_workspace_size(l.attn, n, max_ctx);
}

int check_layer(const li_stack_layer &l, int hidden) {
    if (l.kind == LI_LAYER_DELTANET) {
        if (!l.deltanet || !l.conv_state || !l.state) return LI_ERR_BAD_ARG;
        if (l.deltanet->hidden != hidden) return LI_ERR_BAD_SHAPE;
    } else if (l.kind == LI_LAYER_ATTN) {
        if (!l.attn || !l.k_cache || !l.v_cache) return LI_ERR_BAD_ARG;
        if (l.attn->hidden != hidden) return LI_ERR_BAD_SHAPE;
    } else {
        return LI_ERR_UNSUPPORTED;
    }
    if (!l.ffn.w_gate || !l.ffn.w_up || !l.ffn.w_down || l.ffn.n_inner <= 0) return LI_ERR_BAD_ARG;
    if (l.ffn.hidden != hidden) return LI_ERR_BAD_SHAPE;
    return 0;
}

}  // namespace
}  // namespace li

using namespace li;

extern "C" {

size_t li_stack_workspace_size(const li_stack_layer *layers, int n_layers, int n_seqs, int max_ctx,
                               int tp_nranks) {
    if (!layers || n_layers <= 0 || n_seqs <= 0) return 0;
    const int hidden = layers[0].kind == LI_LAYER_DELTANET
                           ? (layers[0].deltanet ? layers[0].deltanet->hidden : 0)
                           : (layers[0].attn ? layers[0].attn->hidden : 0);
    if (hidden <= 0) return 0;
    size_t need = 0;
    for (int i = 0; i < n_layers; ++i) {
        if (check_layer(layers[i], hidden)) return 0;
        const size_t m = mixer_ws(layers[i], n_seqs, max_ctx), f = ffn_ws(layers[i], n_seqs, tp_nranks);
        need = need > m ? need : m;
        need = need > f ? need : f;
    }
    return al256((size_t)n_seqs * hidden * 4) + need;
}

int li_launch_stack_decode(const li_stack_layer *layers, int n_layers, float *x, const int32_t *pos, int n_seqs,
                           int max_ctx, void *tp_comm, int tp_nranks, void *workspace, size_t workspace_bytes,
                           void *stream) {
    if (!layers || n_layers <= 0 || !x || n_seqs < 0 || tp_nranks <= 0) return LI_ERR_BAD_ARG;
    if (n_seqs == 0) return 0;
    const size_t need = li_stack_workspace_size(layers, n_layers, n_seqs, max_ctx, tp_nranks);
    if (need == 0) {
        // the shape check that made the size 0, reported as such
        const int hidden = layers[0].kind == LI_LAYER_DELTANET
                               ? (layers[0].deltanet ? layers[0].deltanet->hidden : 0)
                               : (layers[0].attn ? layers[0].attn->hidden : 0);
        if (hidden <= 0) return LI_ERR_BAD_ARG;
        for (int i = 0; i < n_layers; ++i)
            if (const int rc = check_layer(layers[i], hidden)) return rc;
        return LI_ERR_BAD_SHAPE;
    }
    if (!workspace || workspace_bytes < need) return LI_ERR_WORKSPACE;
    if (!aligned16(workspace) || !aligned16(x)) return LI_ERR_MISALIGNED;
    const int hidden = layers[0].kind == LI_LAYER_DELTANET ? layers[0].deltanet->hidden : layers[0].attn->hidden;
    const int64_t n = (int64_t)n_seqs * hidden;
    float *t = reinterpret_cast<float *>(workspace);
    char *ws = reinterpret_cast<char *>(workspace) + al256((size_t)n * 4);
    const size_t ws_bytes = workspace_bytes - al256((size_t)n * 4);
    int rc;
    // The residual adds ride on the output projections: each mixer and each
    // unsharded FFN adds its result into x (x += f(x)); the sharded FFN's
    // reduce-scatter lands in t, added by a kernel of its own.
    for (int i = 0; i < n_layers; ++i) {
        const li_stack_layer &l = layers[i];
        if (l.kind == LI_LAYER_DELTANET)
            rc = deltanet_layer_decode_residual(l.deltanet, x, x, l.conv_state, l.state, n_seqs, ws, ws_bytes, stream);
        else
            rc = attn_layer_decode_residual(l.attn, x, x, l.k_cache, l.v_cache, pos, n_seqs, max_ctx, ws, ws_bytes,
                                            stream);
        if (rc) return rc;
        if (tp_nranks > 1) {
            rc = li_launch_ffn_q_tp(l.ffn.wtype, x, l.ffn.norm_w, l.ffn.w_gate, l.ffn.w_up, l.ffn.w_down, t, hidden,
                                    l.ffn.n_inner, n_seqs, l.ffn.eps, tp_comm, tp_nranks, ws, ws_bytes, stream);
            if (!rc) rc = li_launch_add_f32(x, x, t, n, stream);
        } else {
            rc = fused_ffn_q_residual(l.ffn.wtype, x, l.ffn.norm_w, l.ffn.w_gate, l.ffn.w_up, l.ffn.w_down, x, hidden,
                                      l.ffn.n_inner, n_seqs, l.ffn.eps, ws, ws_bytes, stream);
        }
        if (rc) return rc;
    }
    return 0;
}

}  // extern "C"
