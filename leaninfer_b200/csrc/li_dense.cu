// Dense-weight (fp32 / fp16) entries of the reference ABI:
//   li_launch_fused_rms_norm_matmul_f32   (reference cuda/leaninfer-fused-ffn.cu:259-268)
//   li_launch_fused_rms_norm_swiglu_f32   (reference cuda/leaninfer-fused-ffn.cu:270-280)
//   li_launch_fused_rms_norm_swiglu_f16   (reference cuda/leaninfer-fused-ffn.cu:282-292)
//   li_launch_fused_rms_norm_qkv_f32      (reference cuda/leaninfer-fused-deltanet.cu:306-327)
//   li_launch_fused_rms_norm_silu_gate_f32 (reference cuda/leaninfer-fused-gate.cu:92-99)
//
// One kernel template serves the projections: each CTA normalises x into
// shared memory once, then its warps stream weight rows with 16-byte
// read-only loads (4 fp32 or 8 fp16 per lane per load, four loads in flight)
// and reduce with xor-shuffles. The grid is sized to the SM count so the
// RMSNorm prologue runs once per resident CTA rather than once per 8 rows.
#include "li_common.cuh"

LI_DEFINE_TU_STATUS(dense)

namespace li {
namespace {

constexpr int kDenseThreads = 256;
constexpr int kDenseWarps = kDenseThreads / kWarp;

enum DenseMode { kPlain = 0, kSwiGLU = 1 };

struct DenseArgs {
    const float *x;
    const float *gamma;
    const void *W[3];
    float *dst[3];
    int rows[3];        // rows of each matrix (kPlain); rows[0] for kSwiGLU
    int n_mat;
    int K;
    float eps;
};

__device__ __forceinline__ float4 ldg_stream4(const float4 *p) {
    float4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ uint4 ldg_stream_u4(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// RMSNorm of one row of x into shared memory; returns after a CTA barrier.
// round_half: store fp32(fp16(x_norm)) (the reference f16 kernel keeps x_norm
// as half in shared memory, cuda/leaninfer-fused-ffn.cu:230).
__device__ void rmsnorm_to_smem(const float *x, const float *gamma, float *xs, int K,
                                float eps, bool round_half, float *red) {
    float sq = 0.f;
    for (int k = threadIdx.x; k < K; k += blockDim.x) {
        const float v = x[k];
        sq = fmaf(v, v, sq);
    }
    sq = warp_sum(sq);
    const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
    if (lane == 0) red[warp] = sq;
    __syncthreads();
    float tot = 0.f;
    for (int w = 0; w < (int)(blockDim.x / kWarp); ++w) tot += red[w];
    const float r = rsqrtf(tot / (float)K + eps);
    for (int k = threadIdx.x; k < K; k += blockDim.x) {
        float v = x[k] * gamma[k] * r;
        if (round_half) v = __half2float(__float2half(v));
        xs[k] = v;
    }
    __syncthreads();
}

// Dot of one weight row with x_norm (shared), fp32 weights, vectorised.
template <bool VEC>
__device__ __forceinline__ float row_dot_f32(const float *w, const float *xs, int K, int lane) {
    float acc = 0.f;
    if (VEC) {
        const float4 *w4 = reinterpret_cast<const float4 *>(w);
        const float4 *x4 = reinterpret_cast<const float4 *>(xs);
        const int K4 = K >> 2;
        int i = lane;
        for (; i + 3 * kWarp < K4; i += 4 * kWarp) {
            float4 a[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) a[u] = ldg_stream4(w4 + i + u * kWarp);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const float4 xv = x4[i + u * kWarp];
                acc = fmaf(a[u].x, xv.x, acc);
                acc = fmaf(a[u].y, xv.y, acc);
                acc = fmaf(a[u].z, xv.z, acc);
                acc = fmaf(a[u].w, xv.w, acc);
            }
        }
        for (; i < K4; i += kWarp) {
            const float4 a = ldg_stream4(w4 + i);
            const float4 xv = x4[i];
            acc = fmaf(a.x, xv.x, acc);
            acc = fmaf(a.y, xv.y, acc);
            acc = fmaf(a.z, xv.z, acc);
            acc = fmaf(a.w, xv.w, acc);
        }
    } else {
        for (int k = lane; k < K; k += kWarp) acc = fmaf(__ldg(w + k), xs[k], acc);
    }
    return warp_sum(acc);
}

// Same with fp16 weights (8 per 16-byte load).
template <bool VEC>
__device__ __forceinline__ float row_dot_f16(const __half *w, const float *xs, int K, int lane) {
    float acc = 0.f;
    if (VEC) {
        const int K8 = K >> 3;
        const float4 *x4 = reinterpret_cast<const float4 *>(xs);
        int i = lane;
        for (; i + kWarp < K8; i += 2 * kWarp) {
            uint4 a[2];
#pragma unroll
            for (int u = 0; u < 2; ++u) a[u] = ldg_stream_u4(w + 8 * (i + u * kWarp));
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const float4 x0 = x4[2 * (i + u * kWarp)], x1 = x4[2 * (i + u * kWarp) + 1];
                const float2 f0 = __half22float2(*reinterpret_cast<const __half2 *>(&a[u].x));
                const float2 f1 = __half22float2(*reinterpret_cast<const __half2 *>(&a[u].y));
                const float2 f2 = __half22float2(*reinterpret_cast<const __half2 *>(&a[u].z));
                const float2 f3 = __half22float2(*reinterpret_cast<const __half2 *>(&a[u].w));
                acc = fmaf(f0.x, x0.x, acc); acc = fmaf(f0.y, x0.y, acc);
                acc = fmaf(f1.x, x0.z, acc); acc = fmaf(f1.y, x0.w, acc);
                acc = fmaf(f2.x, x1.x, acc); acc = fmaf(f2.y, x1.y, acc);
                acc = fmaf(f3.x, x1.z, acc); acc = fmaf(f3.y, x1.w, acc);
            }
        }
        for (; i < K8; i += kWarp) {
            const uint4 a = ldg_stream_u4(w + 8 * i);
            const float4 x0 = x4[2 * i], x1 = x4[2 * i + 1];
            const float2 f0 = __half22float2(*reinterpret_cast<const __half2 *>(&a.x));
            const float2 f1 = __half22float2(*reinterpret_cast<const __half2 *>(&a.y));
            const float2 f2 = __half22float2(*reinterpret_cast<const __half2 *>(&a.z));
            const float2 f3 = __half22float2(*reinterpret_cast<const __half2 *>(&a.w));
            acc = fmaf(f0.x, x0.x, acc); acc = fmaf(f0.y, x0.y, acc);
            acc = fmaf(f1.x, x0.z, acc); acc = fmaf(f1.y, x0.w, acc);
            acc = fmaf(f2.x, x1.x, acc); acc = fmaf(f2.y, x1.y, acc);
            acc = fmaf(f3.x, x1.z, acc); acc = fmaf(f3.y, x1.w, acc);
        }
    } else {
        for (int k = lane; k < K; k += kWarp) acc = fmaf(__half2float(w[k]), xs[k], acc);
    }
    return warp_sum(acc);
}

template <typename WT, int MODE, bool VEC>
__global__ void __launch_bounds__(kDenseThreads)
dense_gemv_kernel(DenseArgs a) {
    extern __shared__ float4 smem4[];
    float *xs = reinterpret_cast<float *>(smem4);
    __shared__ float red[kDenseWarps];
    rmsnorm_to_smem(a.x, a.gamma, xs, a.K, a.eps, sizeof(WT) == 2, red);

    const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
    const int total = MODE == kSwiGLU ? a.rows[0] : a.rows[0] + a.rows[1] + a.rows[2];
    const int stride = gridDim.x * kDenseWarps;
    for (int row = blockIdx.x * kDenseWarps + warp; row < total; row += stride) {
        if (MODE == kSwiGLU) {
            const WT *wg = reinterpret_cast<const WT *>(a.W[0]) + (size_t)row * a.K;
            const WT *wu = reinterpret_cast<const WT *>(a.W[1]) + (size_t)row * a.K;
            float g, u;
            if (sizeof(WT) == 4) {
                g = row_dot_f32<VEC>(reinterpret_cast<const float *>(wg), xs, a.K, lane);
                u = row_dot_f32<VEC>(reinterpret_cast<const float *>(wu), xs, a.K, lane);
            } else {
                g = row_dot_f16<VEC>(reinterpret_cast<const __half *>(wg), xs, a.K, lane);
                u = row_dot_f16<VEC>(reinterpret_cast<const __half *>(wu), xs, a.K, lane);
            }
            if (lane == 0) a.dst[0][row] = silu(g) * u;
        } else {
            int m = 0, r = row;
            while (m < 2 && r >= a.rows[m]) r -= a.rows[m++];
            const WT *w = reinterpret_cast<const WT *>(a.W[m]) + (size_t)r * a.K;
            float acc;
            if (sizeof(WT) == 4)
                acc = row_dot_f32<VEC>(reinterpret_cast<const float *>(w), xs, a.K, lane);
            else
                acc = row_dot_f16<VEC>(reinterpret_cast<const __half *>(w), xs, a.K, lane);
            if (lane == 0) a.dst[m][r] = acc;
        }
    }
}

// li_launch_fused_rms_norm_qkv_f32 with W_ptrs / dst_ptrs in device memory
// (the reference's comment at cuda/leaninfer-fused-deltanet.cu:304-317 asks
// callers for device-side pointer arrays): the kernel reads the six pointers
// when it runs, so a graph replay sees the arrays' contents at replay time.
// Alignment is known only then, so each row picks the vector or scalar loop;
// a null pointer makes the CTA skip its work and raise LI_ERR_BAD_ARG on the
// device flag.
__global__ void __launch_bounds__(kDenseThreads)
dense_qkv_devptr_kernel(const float *x, const float *gamma, const float *const *W_ptrs, float *const *dst_ptrs,
                        int N, int K, float eps) {
    extern __shared__ float4 smem4[];
    float *xs = reinterpret_cast<float *>(smem4);
    __shared__ float red[kDenseWarps];
    const float *W[3];
    float *dst[3];
    bool ok = true, vec = (K & 3) == 0;
#pragma unroll
    for (int m = 0; m < 3; ++m) {
        W[m] = W_ptrs[m];
        dst[m] = dst_ptrs[m];
        ok = ok && W[m] && dst[m];
        vec = vec && ((uintptr_t)W[m] & 15u) == 0;
    }
    if (!ok) {
        if (threadIdx.x == 0) atomicExch(&g_device_error, LI_ERR_BAD_ARG);
        return;
    }
    rmsnorm_to_smem(x, gamma, xs, K, eps, false, red);
    const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
    const int stride = gridDim.x * kDenseWarps;
    for (int row = blockIdx.x * kDenseWarps + warp; row < 3 * N; row += stride) {
        const int m = row / N, r = row - m * N;
        const float *w = (m == 0 ? W[0] : m == 1 ? W[1] : W[2]) + (size_t)r * K;
        const float acc = vec ? row_dot_f32<true>(w, xs, K, lane) : row_dot_f32<false>(w, xs, K, lane);
        if (lane == 0) (m == 0 ? dst[0] : m == 1 ? dst[1] : dst[2])[r] = acc;
    }
}

template <typename WT, int MODE, bool VEC>
int launch_dense_t(const DenseArgs &a, cudaStream_t stream) {
    const size_t smem = (size_t)a.K * sizeof(float);
    auto kern = dense_gemv_kernel<WT, MODE, VEC>;
    if (smem > 48 * 1024) {
        const cudaError_t e =
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return (int)e;
    }
    const int total = MODE == kSwiGLU ? a.rows[0] : a.rows[0] + a.rows[1] + a.rows[2];
    const int want = (total + kDenseWarps - 1) / kDenseWarps;
    const int grid = want < num_sms() * 4 ? want : num_sms() * 4;
    kern<<<grid, kDenseThreads, smem, stream>>>(a);
    return launch_status();
}

template <typename WT, int MODE>
int launch_dense(const DenseArgs &a, cudaStream_t stream) {
    constexpr int vec = 16 / sizeof(WT);
    bool ok = (a.K % vec) == 0;
    for (int m = 0; m < (MODE == kSwiGLU ? 2 : a.n_mat); ++m) ok = ok && aligned16(a.W[m]);
    return ok ? launch_dense_t<WT, MODE, true>(a, stream) : launch_dense_t<WT, MODE, false>(a, stream);
}

constexpr int kMaxDenseK = (227 * 1024) / 4;

int check_dense(const DenseArgs &a, int n_w) {
    if (!a.x || !a.gamma || a.K <= 0) return LI_ERR_BAD_ARG;
    if (a.K > kMaxDenseK) return LI_ERR_BAD_SHAPE;
    for (int m = 0; m < n_w; ++m)
        if (!a.W[m]) return LI_ERR_BAD_ARG;
    return 0;
}

// ---------------------------------------------------------------------------
// Gated RMSNorm, one warp per row (reference cuda/leaninfer-fused-gate.cu:39-85
// uses a 256-thread block per 128-wide row; a warp is enough for a row).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256)
silu_gate_kernel(const float *__restrict__ o, const float *__restrict__ z,
                 const float *__restrict__ gamma, float *__restrict__ dst, int K, int n_rows,
                 float eps) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) / kWarp;
    const int lane = threadIdx.x % kWarp;
    if (warp >= n_rows) return;
    const float *orow = o + (size_t)warp * K;
    const float *zrow = z + (size_t)warp * K;
    float *drow = dst + (size_t)warp * K;
    float sq = 0.f;
    for (int k = lane; k < K; k += kWarp) sq = fmaf(orow[k], orow[k], sq);
    const float r = rsqrtf(warp_sum(sq) / (float)K + eps);
    for (int k = lane; k < K; k += kWarp) drow[k] = silu(zrow[k]) * (orow[k] * gamma[k] * r);
}

}  // namespace
}  // namespace li

using namespace li;

extern "C" {

void li_launch_fused_rms_norm_matmul_f32(const float *x, const float *gamma, const float *W,
                                         float *dst, int K, int N, float eps, void *stream) {
    DenseArgs a = {};
    a.x = x; a.gamma = gamma; a.W[0] = W; a.dst[0] = dst; a.rows[0] = N; a.n_mat = 1;
    a.K = K; a.eps = eps;
    int rc = check_dense(a, 1);
    if (!rc && (!dst || N < 0)) rc = LI_ERR_BAD_ARG;
    if (!rc && N > 0) rc = launch_dense<float, kPlain>(a, (cudaStream_t)stream);
    set_last_error(rc);
}

void li_launch_fused_rms_norm_swiglu_f32(const float *x, const float *gamma, const float *W_gate,
                                         const float *W_up, float *hidden, int K, int N,
                                         float eps, void *stream) {
    DenseArgs a = {};
    a.x = x; a.gamma = gamma; a.W[0] = W_gate; a.W[1] = W_up; a.dst[0] = hidden;
    a.rows[0] = N; a.n_mat = 2; a.K = K; a.eps = eps;
    int rc = check_dense(a, 2);
    if (!rc && (!hidden || N < 0)) rc = LI_ERR_BAD_ARG;
    if (!rc && N > 0) rc = launch_dense<float, kSwiGLU>(a, (cudaStream_t)stream);
    set_last_error(rc);
}

void li_launch_fused_rms_norm_swiglu_f16(const float *x, const float *gamma, const void *W_gate,
                                         const void *W_up, float *hidden, int K, int N, float eps,
                                         void *stream) {
    DenseArgs a = {};
    a.x = x; a.gamma = gamma; a.W[0] = W_gate; a.W[1] = W_up; a.dst[0] = hidden;
    a.rows[0] = N; a.n_mat = 2; a.K = K; a.eps = eps;
    int rc = check_dense(a, 2);
    if (!rc && (!hidden || N < 0)) rc = LI_ERR_BAD_ARG;
    if (!rc && N > 0) rc = launch_dense<__half, kSwiGLU>(a, (cudaStream_t)stream);
    set_last_error(rc);
}

void li_launch_fused_rms_norm_qkv_f32(const float *x, const float *gamma,
                                      const float *const *W_ptrs, float *const *dst_ptrs,
                                      int K, int N_OUT, float eps, void *stream) {
    int rc = (!W_ptrs || !dst_ptrs) ? LI_ERR_BAD_ARG : 0;
    // Where do the two pointer arrays live? Host arrays (pageable or pinned)
    // are read here, at launch; device (or managed) arrays are read by the
    // kernel. Both arrays must live on the same side.
    int on_device = -1;
    for (const void *arr : {(const void *)W_ptrs, (const void *)dst_ptrs}) {
        if (rc) break;
        cudaPointerAttributes attr;
        int dev_side = 0;
        if (cudaPointerGetAttributes(&attr, arr) == cudaSuccess)
            dev_side = attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged;
        else
            cudaGetLastError();   // an unknown pointer is a plain host pointer
        if (on_device >= 0 && on_device != dev_side) rc = LI_ERR_BAD_ARG;
        on_device = dev_side;
    }
    if (!rc && on_device == 1) {
        if (!x || !gamma || K <= 0 || N_OUT < 0) rc = LI_ERR_BAD_ARG;
        else if (K > kMaxDenseK) rc = LI_ERR_BAD_SHAPE;
        if (!rc && N_OUT > 0) {
            const size_t smem = (size_t)K * sizeof(float);
            if (smem > 48 * 1024) {
                const cudaError_t e = cudaFuncSetAttribute(dense_qkv_devptr_kernel,
                                                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
                if (e != cudaSuccess) rc = (int)e;
            }
            if (!rc) {
                const int want = (3 * N_OUT + kDenseWarps - 1) / kDenseWarps;
                const int grid = want < num_sms() * 4 ? want : num_sms() * 4;
                dense_qkv_devptr_kernel<<<grid, kDenseThreads, smem, (cudaStream_t)stream>>>(
                    x, gamma, W_ptrs, dst_ptrs, N_OUT, K, eps);
                rc = launch_status();
            }
        }
        set_last_error(rc);
        return;
    }
    DenseArgs a = {};
    if (!rc) {
        a.x = x; a.gamma = gamma; a.n_mat = 3; a.K = K; a.eps = eps;
        for (int m = 0; m < 3; ++m) {
            a.W[m] = W_ptrs[m];
            a.dst[m] = dst_ptrs[m];
            a.rows[m] = N_OUT;
            if (!a.dst[m]) rc = LI_ERR_BAD_ARG;
        }
        if (!rc) rc = check_dense(a, 3);
        if (!rc && N_OUT < 0) rc = LI_ERR_BAD_ARG;
    }
    if (!rc && N_OUT > 0) rc = launch_dense<float, kPlain>(a, (cudaStream_t)stream);
    set_last_error(rc);
}

void li_launch_fused_rms_norm_silu_gate_f32(const float *output, const float *z,
                                            const float *gamma, float *dst, int K, int n_rows,
                                            float eps, void *stream) {
    int rc = 0;
    if (!output || !z || !gamma || !dst || K <= 0 || n_rows < 0) rc = LI_ERR_BAD_ARG;
    if (!rc && n_rows > 0) {
        const int blocks = (n_rows + 7) / 8;
        silu_gate_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(output, z, gamma, dst, K,
                                                                   n_rows, eps);
        rc = launch_status();
    }
    set_last_error(rc);
}

}  // extern "C"
