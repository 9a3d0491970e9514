// Host interface of the tcgen05 batched-decode projections (li_tcgemm.cu).
#pragma once
#include <stddef.h>
#include <cuda_runtime.h>

namespace li {

// Batch rows below this use the SIMT GEMV (li_qgemv.cu), which reads the
// weights once per row; at and above it the dense contraction goes to the
// tensor cores (measured on B200: SIMT 44.6 µs vs tensor 51 µs per layer step
// at 2 rows, 59.9 vs 52 at 3, 74 vs 52 at 4).
constexpr int kTcMinRows = 3;

enum TcEpilogue {
    kTcStore = 0,    // dst[seg][b][row] = acc
    kTcSwiGLU = 1,   // dst[0][b][row] = silu(acc_gate) * acc_up (two weight matrices)
    kTcConv = 2,     // DeltaNet in-projection: conv1d(4)+SiLU for row < conv_channels
};

struct TcArgs {
    int wtype, epi;
    int K;                 // reduction length (multiple of 256)
    int total_rows;        // weight rows (output features) over all segments
    int B;                 // batch rows of X
    const void *W[3];      // kTcSwiGLU: W[0] gate, W[1] up (one segment)
    int n_seg;
    int seg_rows[3];
    float *dst[3];
    int dst_stride[3];
    const __half *X16;     // [B][K] f16 operand (K-major)
    const float *xscale;   // [B] output multiplier per batch row, or nullptr (1)
    const float *conv_w;   // kTcConv
    float *conv_state;
    int conv_channels;
};

// x[b] (fp32) -> X16[b] = f16(rmsnorm?(x[b]) / s_b), xscale[b] = s_b (a power
// of two that keeps the row inside f16 range). gamma == nullptr: no norm.
int tc_prep_launch(const float *x, int x_stride, const float *gamma, float eps, int B, int K,
                   __half *X16, float *xscale, cudaStream_t stream, bool pdl);

// One launch covers all batch rows (up to 256); returns LI_ERR_* / cudaError_t.
// kTcStore launches may split K over several CTAs per tile and then ADD into
// dst: the caller zeroes dst first when tc_gemm_splits_k(a) is true.
int tc_gemm_launch(const TcArgs &a, cudaStream_t stream, bool pdl);
bool tc_gemm_splits_k(const TcArgs &a);

}  // namespace li
