// The prefill's output stage on the tensor cores: the gated RMSNorm of the
// head outputs written as bf16, and a plain bf16 GEMM C[M][N] (fp32) =
// A[M][K] . W[N][K]^T (the 4096 -> 4096 out-projection over the prompt's
// tokens).
//
// GEMM: one CTA per 128 x 256 output tile, 6 warps:
//   warp 0 lane 0: TMA producer (2-D tiled, 128-byte swizzle) of A [128][64]
//       and W [256][64] k-steps into a 4-stage ring (48 KB per stage);
//   warp 1: allocates 256 TMEM columns; lane 0 issues tcgen05.mma
//       kind::f16 (bf16 x bf16, fp32 accumulate), M = 128, N = 256, four
//       K = 16 steps per stage, and commits stage releases;
//   warps 2-5: epilogue, one TMEM lane quarter each (warp w serves lanes
//       32 (w % 4) ..), tcgen05.ld 32 columns at a time, float4 stores.
// All mbarrier waits are bounded (a timeout raises the device flag, drains
// the copies in flight and frees the TMEM after the MMAs).
#include "li_common.cuh"
#include "li_tc.cuh"

#include <cuda.h>
#include <cuda_bf16.h>
#include <mutex>

LI_DEFINE_TU_STATUS(gemm_bf16)

namespace li {
namespace {

constexpr int kGM = 128, kGN = 256, kGK = 64, kGStages = 4;
constexpr uint32_t kGA = kGM * kGK * 2, kGB = kGN * kGK * 2, kGStage = kGA + kGB;   // 16 KB, 32 KB
constexpr size_t kGSmem = (size_t)kGStages * kGStage + 1024 + 256;

__device__ __forceinline__ void tma_2d(void *dst, const CUtensorMap *m, int x, int y, uint64_t *bar) {
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
                 " [%0], [%1, {%2, %3}], [%4];"
                 ::"r"(smem_addr(dst)), "l"(m), "r"(x), "r"(y), "r"(smem_addr(bar)) : "memory");
}

__global__ void __launch_bounds__(192, 1)
gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW, float *C,
                 int M, int N, int K) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *sm = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    uint64_t *full = reinterpret_cast<uint64_t *>(sm + kGStages * kGStage);
    uint64_t *empty = full + kGStages;
    uint64_t *acc = empty + kGStages;
    uint32_t *holder = reinterpret_cast<uint32_t *>(acc + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(holder + 1);

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int n0 = blockIdx.x * kGN, m0 = blockIdx.y * kGM;
    const int nk = K / kGK;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kGStages; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        mbar_init(acc, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(holder, 256);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *holder;

    if (warp == 0 && lane == 0) {
        int issued = 0;
        for (int kb = 0; kb < nk; ++kb) {
            const int s = kb % kGStages;
            if (kb >= kGStages && !mbar_wait(&empty[s], (uint32_t)(((kb / kGStages) - 1) & 1))) {
                *abort_flag = 1;
                break;
            }
            uint8_t *st = sm + (size_t)s * kGStage;
            mbar_arrive_expect_tx(&full[s], kGStage);
            tma_2d(st, &tmA, kb * kGK, m0, &full[s]);
            tma_2d(st + kGA, &tmW, kb * kGK, n0, &full[s]);
            issued = kb + 1;
        }
        for (int kb = issued - kGStages < 0 ? 0 : issued - kGStages; kb < issued; ++kb)
            mbar_wait(&full[kb % kGStages], (uint32_t)((kb / kGStages) & 1));
    } else if (warp == 1 && lane == 0) {
        const uint32_t idesc = idesc_kf16(kGM, kGN, true);
        for (int kb = 0; kb < nk; ++kb) {
            const int s = kb % kGStages;
            if (*abort_flag || !mbar_wait(&full[s], (uint32_t)((kb / kGStages) & 1))) {
                *abort_flag = 1;
                break;
            }
            tc_fence_after();
            const uint8_t *st = sm + (size_t)s * kGStage;
            const uint64_t da = sw128_desc(smem_addr(st)), dw = sw128_desc(smem_addr(st + kGA));
#pragma unroll
            for (int j = 0; j < 4; ++j) umma_f16(tmem, da + 2 * j, dw + 2 * j, idesc, (kb | j) ? 1u : 0u);
            umma_commit(&empty[s]);
        }
        umma_commit(acc);   // every MMA issued has finished when this arrives
    } else if (warp >= 2) {
        const int q = warp & 3;
        const bool ok = __all_sync(0xffffffffu, mbar_wait(acc, 0u)) && __all_sync(0xffffffffu, *abort_flag == 0);
        tc_fence_after();
        if (ok) {
            const int row = m0 + 32 * q + lane;
            float *crow = C + (size_t)row * N + n0;
            for (int c0 = 0; c0 < kGN; c0 += 32) {
                uint32_t r[32];
                tmem_ld32_nowait(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)c0, r);
                tmem_wait_ld();
                if (row < M) {
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        *reinterpret_cast<float4 *>(crow + c0 + 4 * j) =
                            make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                        __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
                }
            }
        }
    }
    if (*abort_flag && threadIdx.x == 0) atomicExch(&g_device_error, LI_ERR_TIMEOUT);
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        if (*abort_flag && lane == 0) mbar_wait(acc, 0u);
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, 256);
    }
}

// dst[row][k] = bf16( silu(z) * (o * gamma * rsqrt(mean(o^2) + eps)) ), one warp per row, 16-byte
// loads (the arithmetic of the reference's fused gate, cuda/leaninfer-fused-gate.cu:53-85); K % 4 == 0
__global__ void __launch_bounds__(256)
gated_rmsnorm_bf16_kernel(const float *__restrict__ o, const float *__restrict__ z, const float *__restrict__ gamma,
                          __nv_bfloat16 *__restrict__ dst, int K, int64_t n_rows, float eps) {
    const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / kWarp;
    const int lane = threadIdx.x % kWarp;
    if (row >= n_rows) return;
    const float4 *o4 = reinterpret_cast<const float4 *>(o + row * K);
    const float4 *z4 = reinterpret_cast<const float4 *>(z + row * K);
    const float4 *g4 = reinterpret_cast<const float4 *>(gamma);
    const int K4 = K / 4;
    uint2 *d2 = reinterpret_cast<uint2 *>(dst + row * K);
    if (K4 <= kWarp) {
        // one 16-byte chunk per lane (head_dim 128): o is read once
        const bool on = lane < K4;
        const float4 v = on ? __ldcs(o4 + lane) : make_float4(0.f, 0.f, 0.f, 0.f);
        const float4 zz = on ? __ldcs(z4 + lane) : v, g = on ? g4[lane] : v;
        const float r = rsqrtf(warp_sum(fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, v.w * v.w)))) / (float)K + eps);
        if (on) {
            const __nv_bfloat162 a = __floats2bfloat162_rn(silu(zz.x) * (v.x * g.x * r), silu(zz.y) * (v.y * g.y * r));
            const __nv_bfloat162 b = __floats2bfloat162_rn(silu(zz.z) * (v.z * g.z * r), silu(zz.w) * (v.w * g.w * r));
            d2[lane] = make_uint2(*reinterpret_cast<const uint32_t *>(&a), *reinterpret_cast<const uint32_t *>(&b));
        }
        return;
    }
    float sq = 0.f;
    for (int k = lane; k < K4; k += kWarp) {
        const float4 v = o4[k];
        sq = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, sq))));
    }
    const float r = rsqrtf(warp_sum(sq) / (float)K + eps);
    for (int k = lane; k < K4; k += kWarp) {
        const float4 v = o4[k], zz = __ldcs(z4 + k), g = g4[k];
        const __nv_bfloat162 a = __floats2bfloat162_rn(silu(zz.x) * (v.x * g.x * r), silu(zz.y) * (v.y * g.y * r));
        const __nv_bfloat162 b = __floats2bfloat162_rn(silu(zz.z) * (v.z * g.z * r), silu(zz.w) * (v.w * g.w * r));
        d2[k] = make_uint2(*reinterpret_cast<const uint32_t *>(&a), *reinterpret_cast<const uint32_t *>(&b));
    }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encoder() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

int encode_bf16(CUtensorMap *m, const void *base, int inner, int rows, int box_rows) {
    EncodeTiledFn fn = encoder();
    if (!fn) return LI_ERR_UNSUPPORTED;
    const cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)inner * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kGK, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : LI_ERR_BAD_SHAPE;
}

}  // namespace
}  // namespace li

using namespace li;

extern "C" {

int li_launch_gemm_bf16_f32(const void *A, const void *W, float *C, int M, int N, int K, void *stream) {
    if (!A || !W || !C || M < 0 || N < 0 || K < 0) return LI_ERR_BAD_ARG;
    if (M == 0 || N == 0) return 0;
    if (M % kGM || N % kGN || K % kGK || K == 0) return LI_ERR_BAD_SHAPE;
    if (!aligned16(A) || !aligned16(W) || !aligned16(C)) return LI_ERR_MISALIGNED;
    static std::once_flag once;
    static cudaError_t attr = cudaSuccess;
    std::call_once(once, [] {
        attr = cudaFuncSetAttribute(gemm_bf16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGSmem);
    });
    if (attr != cudaSuccess) return (int)attr;
    CUtensorMap ma, mw;
    int rc = encode_bf16(&ma, A, K, M, kGM);
    if (!rc) rc = encode_bf16(&mw, W, K, N, kGN);
    if (rc) return rc;
    gemm_bf16_kernel<<<dim3((unsigned)(N / kGN), (unsigned)(M / kGM)), 192, kGSmem, (cudaStream_t)stream>>>(
        ma, mw, C, M, N, K);
    return launch_status();
}

int li_launch_gated_rmsnorm_bf16(const float *o, const float *z, const float *gamma, void *dst, int K,
                                 int64_t n_rows, float eps, void *stream) {
    if (!o || !z || !gamma || !dst || K <= 0 || n_rows < 0) return LI_ERR_BAD_ARG;
    if (n_rows == 0) return 0;
    if (K % 4) return LI_ERR_BAD_SHAPE;
    if (!aligned16(o) || !aligned16(z) || !aligned16(gamma) || ((uintptr_t)dst & 7u)) return LI_ERR_MISALIGNED;
    const int64_t blocks = (n_rows * kWarp + 255) / 256;
    gated_rmsnorm_bf16_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(o, z, gamma, (__nv_bfloat16 *)dst,
                                                                                  K, n_rows, eps);
    return launch_status();
}

}  // extern "C"
