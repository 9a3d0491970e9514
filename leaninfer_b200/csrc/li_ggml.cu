// ggml-style node dispatch onto the C entries (host code only).
//
// li_ggml_compute_forward reads a node the way a ggml-cuda
// ggml_cuda_compute_forward case does (reference
// scripts/patch_fused_gate.sh:167-204: sources from dst->src[], K from
// src[0]->ne[0], rows from the element count, eps from op_params), checks
// types and contiguous strides, and calls the entry of leaninfer-cuda.h.
// Node layouts are listed in include/leaninfer-ggml.h.
#include "leaninfer-ggml.h"

#include <cstring>

namespace {

int64_t rows_of(const li_ggml_tensor *t) { return t->ne[1] * t->ne[2] * t->ne[3]; }

bool dims_ok(const li_ggml_tensor *t) {
    for (int i = 0; i < LI_GGML_MAX_DIMS; ++i)
        if (t->ne[i] < 1) return false;
    return true;
}

// f32, every stride the contiguous one
bool f32_contiguous(const li_ggml_tensor *t) {
    if (t->type != LI_GGML_TYPE_F32 || !dims_ok(t)) return false;
    size_t s = sizeof(float);
    for (int i = 0; i < LI_GGML_MAX_DIMS; ++i) {
        if (t->ne[i] > 1 && t->nb[i] != s) return false;
        s *= (size_t)t->ne[i];
    }
    return true;
}

// f16, every stride the contiguous one
bool f16_contiguous(const li_ggml_tensor *t) {
    if (t->type != LI_GGML_TYPE_F16 || !dims_ok(t)) return false;
    size_t s = 2;
    for (int i = 0; i < LI_GGML_MAX_DIMS; ++i) {
        if (t->ne[i] > 1 && t->nb[i] != s) return false;
        s *= (size_t)t->ne[i];
    }
    return true;
}

// quantized matrix [k, n] of contiguous rows
bool quant_matrix(const li_ggml_tensor *t, int64_t k, int64_t n) {
    if ((t->type != LI_GGML_TYPE_Q8_0 && t->type != LI_GGML_TYPE_Q4_K) || !dims_ok(t)) return false;
    if (t->ne[0] != k || t->ne[1] != n || t->ne[2] != 1 || t->ne[3] != 1) return false;
    const size_t rb = li_row_bytes(t->type, k);
    return rb != 0 && t->nb[0] == (t->type == LI_GGML_TYPE_Q8_0 ? 34u : 144u) && (n == 1 || t->nb[1] == rb);
}

bool is_quant(const li_ggml_tensor *t) {
    return t && (t->type == LI_GGML_TYPE_Q8_0 || t->type == LI_GGML_TYPE_Q4_K);
}

float param_f32(const li_ggml_tensor *t, int i) {
    float v;
    std::memcpy(&v, &t->op_params[i], sizeof(v));
    return v;
}

bool fits_int(int64_t v) { return v > 0 && v <= 0x7fffffff; }

// the f32 vector [n] (any trailing dims of extent 1)
bool f32_vector(const li_ggml_tensor *t, int64_t n) {
    return t && t->data && f32_contiguous(t) && t->ne[0] == n && rows_of(t) == 1;
}

// li_deltanet_layer from a DELTANET_DECODE node; 0 or a status
int layer_of(const li_ggml_tensor *node, li_deltanet_layer *L, int *n_seqs) {
    for (int i = 0; i < 9; ++i)
        if (!node->src[i] || !node->src[i]->data) return LI_ERR_BAD_ARG;
    const li_ggml_tensor *x = node->src[0], *cs = node->src[1], *st = node->src[2], *win = node->src[3],
                         *cw = node->src[4], *wout = node->src[8], *inw = node->src[9];
    if (!is_quant(win) || !is_quant(wout)) return LI_ERR_UNSUPPORTED;
    if (st->type != LI_GGML_TYPE_F32 && st->type != LI_GGML_TYPE_F16) return LI_ERR_UNSUPPORTED;
    if (!f32_contiguous(x) || !f32_contiguous(node) || !f32_contiguous(cs) || !f32_contiguous(cw) ||
        !(st->type == LI_GGML_TYPE_F32 ? f32_contiguous(st) : f16_contiguous(st)))
        return LI_ERR_BAD_SHAPE;
    const int64_t hidden = x->ne[0], n = rows_of(x);
    const int64_t D = st->ne[0], Hv = st->ne[2], Hk = node->op_params[0];
    if (st->ne[1] != D || st->ne[3] != n || Hk < 1 || Hv % Hk) return LI_ERR_BAD_SHAPE;
    const int64_t C = 2 * Hk * D + Hv * D, NI = C + Hv * D + 2 * Hv;
    if (node->ne[0] != hidden || rows_of(node) != n) return LI_ERR_BAD_SHAPE;
    if (cs->ne[0] != 3 || cs->ne[1] != C || cs->ne[2] * cs->ne[3] != n) return LI_ERR_BAD_SHAPE;
    if (cw->ne[1] != C || rows_of(cw) != C) return LI_ERR_BAD_SHAPE;
    if (!quant_matrix(win, hidden, NI) || !quant_matrix(wout, Hv * D, hidden)) return LI_ERR_BAD_SHAPE;
    if (!f32_vector(node->src[5], Hv) || !f32_vector(node->src[6], Hv) || !f32_vector(node->src[7], D))
        return LI_ERR_BAD_SHAPE;
    if (inw && !f32_vector(inw, hidden)) return LI_ERR_BAD_SHAPE;
    if (!fits_int(hidden) || !fits_int(n) || !fits_int(NI)) return LI_ERR_BAD_SHAPE;
    std::memset(L, 0, sizeof(*L));
    L->hidden = (int)hidden;
    L->n_k_heads = (int)Hk;
    L->n_v_heads = (int)Hv;
    L->head_dim = (int)D;
    L->conv_kernel = (int)cw->ne[0];
    L->repeat_type = node->op_params[1];
    L->w_in_type = win->type;
    L->w_out_type = wout->type;
    L->l2_eps = param_f32(node, 2);
    L->norm_eps = param_f32(node, 3);
    L->in_norm_eps = param_f32(node, 4);
    L->in_norm_w = inw ? (const float *)inw->data : nullptr;
    L->w_in = win->data;
    L->conv_w = (const float *)cw->data;
    L->a_log = (const float *)node->src[5]->data;
    L->dt_bias = (const float *)node->src[6]->data;
    L->norm_w = (const float *)node->src[7]->data;
    L->w_out = wout->data;
    *n_seqs = (int)n;
    return 0;
}

}  // namespace

extern "C" {

size_t li_ggml_workspace_size(const li_ggml_tensor *node) {
    if (!node || node->op != LI_GGML_OP_DELTANET_DECODE) return 0;
    li_deltanet_layer L;
    int n = 0;
    if (layer_of(node, &L, &n)) return 0;
    return li_deltanet_layer_workspace_size(&L, n);
}

int li_ggml_compute_forward(const li_ggml_tensor *node, void *workspace, size_t workspace_bytes,
                            void *stream) {
    if (!node || !node->data) return LI_ERR_BAD_ARG;
    switch (node->op) {
    case LI_GGML_OP_MUL_MAT: {
        const li_ggml_tensor *w = node->src[0], *x = node->src[1];
        if (!w || !x || !w->data || !x->data) return LI_ERR_BAD_ARG;
        if (!is_quant(w)) return LI_ERR_UNSUPPORTED;
        const int64_t K = w->ne[0], N = w->ne[1], M = rows_of(x);
        if (!quant_matrix(w, K, N) || !f32_contiguous(x) || !f32_contiguous(node)) return LI_ERR_BAD_SHAPE;
        if (x->ne[0] != K || node->ne[0] != N || rows_of(node) != M) return LI_ERR_BAD_SHAPE;
        if (!fits_int(K) || !fits_int(N) || !fits_int(M)) return LI_ERR_BAD_SHAPE;
        return li_launch_rms_norm_matmul_q(w->type, (const float *)x->data, nullptr, w->data, (float *)node->data,
                                           (int)K, (int)N, (int)M, 0.f, stream);
    }
    case LI_GGML_OP_FUSED_UP_GATE: {
        const li_ggml_tensor *wu = node->src[0], *wg = node->src[1], *x = node->src[2];
        if (!wu || !wg || !x || !wu->data || !wg->data || !x->data) return LI_ERR_BAD_ARG;
        if (!is_quant(wu) || wg->type != wu->type) return LI_ERR_UNSUPPORTED;
        const int64_t K = wu->ne[0], N = wu->ne[1], M = rows_of(x);
        if (!quant_matrix(wu, K, N) || !quant_matrix(wg, K, N) || !f32_contiguous(x) || !f32_contiguous(node))
            return LI_ERR_BAD_SHAPE;
        if (x->ne[0] != K || node->ne[0] != N || rows_of(node) != M) return LI_ERR_BAD_SHAPE;
        if (!fits_int(K) || !fits_int(N) || !fits_int(M)) return LI_ERR_BAD_SHAPE;
        return li_launch_fused_rms_norm_swiglu_q(wu->type, (const float *)x->data, nullptr, wg->data, wu->data,
                                                 (float *)node->data, (int)K, (int)N, (int)M, 0.f, stream);
    }
    case LI_GGML_OP_FUSED_RMS_SILU_GATE: {
        const li_ggml_tensor *o = node->src[0], *z = node->src[1], *g = node->src[2];
        if (!o || !z || !g || !o->data || !z->data || !g->data) return LI_ERR_BAD_ARG;
        if (!f32_contiguous(o) || !f32_contiguous(z) || !f32_contiguous(node)) return LI_ERR_BAD_SHAPE;
        const int64_t K = o->ne[0], R = rows_of(o);
        for (int i = 0; i < LI_GGML_MAX_DIMS; ++i)
            if (z->ne[i] != o->ne[i] || node->ne[i] != o->ne[i]) return LI_ERR_BAD_SHAPE;
        if (!f32_vector(g, K) || !fits_int(K) || !fits_int(R)) return LI_ERR_BAD_SHAPE;
        li_get_last_error();   // clear
        li_launch_fused_rms_norm_silu_gate_f32((const float *)o->data, (const float *)z->data,
                                               (const float *)g->data, (float *)node->data, (int)K, (int)R,
                                               param_f32(node, 0), stream);
        return li_get_last_error();
    }
    case LI_GGML_OP_DELTANET_DECODE: {
        li_deltanet_layer L;
        int n = 0;
        const int rc = layer_of(node, &L, &n);
        if (rc) return rc;
        if (node->src[2]->type == LI_GGML_TYPE_F16)   // fp16 state storage
            return li_launch_deltanet_layer_decode_f16state(&L, (const float *)node->src[0]->data,
                                                            (float *)node->data, (float *)node->src[1]->data,
                                                            node->src[2]->data, n, workspace, workspace_bytes,
                                                            stream);
        return li_launch_deltanet_layer_decode(&L, (const float *)node->src[0]->data, (float *)node->data,
                                               (float *)node->src[1]->data, (float *)node->src[2]->data, n,
                                               workspace, workspace_bytes, stream);
    }
    default:
        return LI_ERR_UNSUPPORTED;
    }
}

}  // extern "C"
