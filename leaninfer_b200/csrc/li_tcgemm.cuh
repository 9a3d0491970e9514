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
    const __half *X16;     // [B][K] f16 operand (K-major), or tiled (x_npad > 0)
    int x_npad;            // > 0: X16 is tiled for the X-stationary kernel (tiled_x_offset)
    const float *xscale;   // [B] output multiplier per batch row, or nullptr (1)
    const float *conv_w;   // kTcConv
    float *conv_state;
    int conv_channels;
    // fp32 scratch of tc_gemm_partials_bytes() for the X-stationary kernel
    // (batch <= 64); nullptr keeps the one-tile-per-CTA kernel
    float *partials;
    // kTcStore: 1 adds the result to what dst holds (a residual update); a
    // K-split GEMM then adds its partial sums onto dst instead of a zeroed
    // output
    int accumulate;
};

// Tiled X for the X-stationary kernel: [K/64][npad rows][64 k] f16, each
// [npad][64] k-block in the 128-byte-swizzled K-major MMA layout (16-byte
// granule g of row b at granule g ^ (b % 8)), so a k-chunk is one contiguous
// block; rows B .. npad-1 are never written (their products are discarded).
// Element offset of (b, k):
__host__ __device__ inline size_t tiled_x_offset(int b, int k, int npad) {
    return (size_t)(k >> 6) * npad * 64 + (size_t)(b >> 3) * 512 + (b & 7) * 64 + ((((k & 63) >> 3) ^ (b & 7)) << 3) +
           (k & 7);
}

// x[b] (fp32) -> X16[b] = f16(rmsnorm?(x[b]) / s_b), xscale[b] = s_b (a power
// of two that keeps the row inside f16 range). gamma == nullptr: no norm.
// x_npad > 0 writes X16 tiled (tiled_x_offset), else row-major [B][K].
// early_dependents: the kernel lets its dependent launch at entry, for the
// X-stationary GEMM only (tc_gemm_x_stationary), which then streams and
// dequantizes its weights while the prep runs; its reduce kernel waits for it
// before letting anything after it launch.
int tc_prep_launch(const float *x, int x_stride, const float *gamma, float eps, int B, int K,
                   __half *X16, float *xscale, cudaStream_t stream, bool pdl, int x_npad = 0,
                   bool early_dependents = false);

// One launch covers all batch rows (up to 256); returns LI_ERR_* / cudaError_t.
// kTcStore and kTcConv launches may split K over several CTAs per tile and
// then ADD into dst (kTcConv: the raw projections, then a second launch runs
// the conv epilogue over them): the caller zeroes dst first when
// tc_gemm_splits_k(a) is true.
int tc_gemm_launch(const TcArgs &a, cudaStream_t stream, bool pdl);
bool tc_gemm_splits_k(const TcArgs &a);

// Scratch for the per-chunk partial sums of the X-stationary kernel (0 when
// that kernel does not apply to this shape; then partials stay unused).
size_t tc_gemm_partials_bytes(int wtype, int epi, int K, int rows_total, int B);

// Rows of the tiled X (x_npad) the launch with these arguments (X16 and
// x_npad aside) will use the X-stationary kernel with, or 0 when it will not.
int tc_gemm_x_npad(const TcArgs &a);
// True when this GEMM runs on the X-stationary kernel (K chunks + reduce).
bool tc_gemm_x_stationary(const TcArgs &a);

}  // namespace li
