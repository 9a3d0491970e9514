// Host interface of the quantized GEMV stages (li_qgemv.cu), shared with the
// DeltaNet layer decode (li_deltanet.cu).
#pragma once
#include <stddef.h>
#include <cuda_runtime.h>

namespace li {

enum QEpilogue {
    kEpiStore = 0,   // dst[seg][b][row] = acc
    kEpiSwiGLU = 1,  // dst[0][b][row] = silu(acc_gate) * acc_up
    kEpiConv = 2,    // DeltaNet in-projection: conv1d(4)+SiLU for row < conv_channels
};

struct QGemvPlan {
    int U, UP, RP, R, SR, S, XB, threads;
    int total_rows;
    size_t row_bytes, smem;
};

struct QGemvArgs {
    int wtype, epi;
    QGemvPlan plan;
    const float *x;          // [n_rows][x_stride]
    int x_stride;
    const float *gamma;      // RMSNorm weight or nullptr
    int K;
    float eps;
    int n_seg;               // weight segments in the output row space
    const void *W[3];        // kEpiSwiGLU: W[0] gate, W[1] up
    int seg_rows[3];
    float *dst[3];
    int dst_stride[3];
    // kEpiConv
    const float *conv_w;     // [conv_channels][4]
    float *conv_state;       // [n_rows][conv_channels][3]
    int conv_channels;
    // kEpiStore: 1 adds the result to what dst holds (a residual update,
    // dst[b][row] += acc) instead of overwriting it
    int accumulate;
};

int qgemv_plan(int wtype, int K, int total_rows, int epi, QGemvPlan *p);
int qgemv_launch(const QGemvArgs &a, int n_rows, cudaStream_t stream, bool pdl);
// True when n_rows x rows of this shape take the few-row kernel (weights in
// registers, every x row per weight load; x and gamma 16-byte aligned, x
// rows a multiple of 4 floats apart).
bool qgemv_few_rows(int wtype, int K, int n_rows);

}  // namespace li
