// Shared device and host helpers of the LeanInfer B200 kernels (sm_100a).
//
// Block formats (ggml, as decoded by gguf-py 0.19.0 quants.py):
//   Q8_0  34 B / 32 values : fp16 d | int8 q[32]              v = d*q
//   Q4_K 144 B / 256 values: fp16 d | fp16 dmin | 12 B 6-bit scales/mins |
//                            128 B nibbles; sub-block 2i = low nibbles of
//                            qs[32i..32i+31], 2i+1 = their high nibbles;
//                            v = d*sc_j*q - dmin*m_j
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "leaninfer-cuda.h"

namespace li {

constexpr int kWarp = 32;
constexpr int kQ80Bytes = 34;
constexpr int kQ4KBytes = 144;

// ---------------------------------------------------------------------------
// Host-side status plumbing (li_abi.cu)
// ---------------------------------------------------------------------------
void set_last_error(int code);                 // legacy void entries
int  num_sms();                                // SMs of the current device
int  launch_status();                          // cudaGetLastError as int

// Residual forms of the layer entries, for the layer stack: y += layer(x),
// where y may be x itself (every read of x precedes the first write of y in
// stream order). The output projection adds its result to y instead of
// storing it (a K-split projection adds its partial sums onto y instead of
// a zeroed output), so the stack needs no separate residual-add kernel.
int deltanet_layer_decode_residual(const li_deltanet_layer *L, const float *x, float *y, float *conv_state,
                                   float *state, int n_seqs, void *workspace, size_t workspace_bytes, void *stream);
int attn_layer_decode_residual(const li_attn_layer *L, const float *x, float *y, void *k_cache, void *v_cache,
                               const int32_t *pos, int n_seqs, int max_ctx, void *workspace, size_t workspace_bytes,
                               void *stream);
int fused_ffn_q_residual(int wtype, const float *x, const float *gamma, const void *Wg, const void *Wu,
                         const void *Wd, float *y, int K, int N, int n_rows, float eps, void *workspace,
                         size_t workspace_bytes, void *stream);

// Device-side failure flag (a bounded wait that gave up). Each translation
// unit has its own copy (internal linkage, no relocatable device code); each
// defines a host reader with LI_DEFINE_TU_STATUS, and li_device_status()
// reads and clears all of them.
static __device__ int g_device_error;

#define LI_DEFINE_TU_STATUS(name)                                              \
    int li_tu_status_##name(int clear) {                                       \
        int v = 0;                                                             \
        if (cudaMemcpyFromSymbol(&v, li::g_device_error, sizeof(int)) != cudaSuccess) \
            return (int)cudaGetLastError();                                    \
        if (clear && v) {                                                      \
            int z = 0;                                                         \
            cudaMemcpyToSymbol(li::g_device_error, &z, sizeof(int));           \
        }                                                                      \
        return v;                                                              \
    }

// ---------------------------------------------------------------------------
// Arithmetic helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float silu(float x) { return x / (1.0f + expf(-x)); }

__device__ __forceinline__ float sigmoid(float x) { return 1.0f / (1.0f + expf(-x)); }

__device__ __forceinline__ float softplus(float x) {
    return x > 20.0f ? x : log1pf(expf(x));
}

__device__ __forceinline__ float half_bits_to_float(uint32_t h16) {
    return __half2float(__ushort_as_half((unsigned short)(h16 & 0xffffu)));
}

// Float with value (2^23 + b) built from one byte b of `w` by a byte permute;
// subtracting 2^23 gives b exactly (0 <= b < 256).
__device__ __forceinline__ float byte_to_float(uint32_t w, int b) {
    const uint32_t bits = __byte_perm(w, 0x4B000000u, 0x7540u | (uint32_t)b);
    return __uint_as_float(bits) - 8388608.0f;
}

// Q4_K scale and min of sub-block j (0..7) from the 12 scale bytes held in
// three little-endian words s0 (bytes 0-3), s1 (4-7), s2 (8-11).
__device__ __forceinline__ void q4k_scale_min(uint32_t s0, uint32_t s1, uint32_t s2,
                                              int j, float &sc, float &mn) {
    if (j < 4) {
        sc = (float)((s0 >> (8 * j)) & 63u);
        mn = (float)((s1 >> (8 * j)) & 63u);
    } else {
        const int i = j - 4;
        const uint32_t a = (s2 >> (8 * i)) & 0xffu;   // byte j+4
        const uint32_t hs = (s0 >> (8 * i + 6)) & 3u;  // top bits of byte j-4
        const uint32_t hm = (s1 >> (8 * i + 6)) & 3u;  // top bits of byte j
        sc = (float)((a & 0x0fu) | (hs << 4));
        mn = (float)((a >> 4) | (hm << 4));
    }
}

// ---------------------------------------------------------------------------
// mbarrier + bulk async copy (TMA engine, 1-D form). All waits are bounded:
// after ~kWaitNs of polling the wait gives up, raises g_device_error and
// returns false.
// ---------------------------------------------------------------------------
constexpr unsigned long long kWaitNs = 1000ull * 1000ull * 1000ull;   // 1 s

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_shared() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;"
                 ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity), "r"(10000000u)
        : "memory");
    return ok != 0;
}

// Wait for phase `parity` of `bar` for at most limit_ns of %globaltimer.
// On timeout it raises LI_ERR_TIMEOUT on the device flag and returns false.
__device__ __forceinline__ bool mbar_wait_for(uint64_t *bar, uint32_t parity, unsigned long long limit_ns) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = global_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (global_ns() - t0 > limit_ns) {
            atomicExch(&g_device_error, LI_ERR_TIMEOUT);
            return false;
        }
    }
    return true;
}

// Bounded wait (kWaitNs) for phase `parity` of `bar`. Returns false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
    return mbar_wait_for(bar, parity, kWaitNs);
}

// Bulk copy of `bytes` (multiple of 16, both addresses 16-byte aligned)
// from global to this CTA's shared memory; completion is signalled on `bar`.
__device__ __forceinline__ void bulk_g2s(void *smem_dst, const void *gsrc, uint32_t bytes,
                                         uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(smem_addr(smem_dst)), "l"(gsrc), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// Hint: bring `bytes` (a multiple of 16, 16-byte aligned) of global memory into
// L2 ahead of use (bulk async, nothing to wait for).
__device__ __forceinline__ void bulk_prefetch_l2(const void *gsrc, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(gsrc), "r"(bytes) : "memory");
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch (sm_90+): a kernel launched with the
// programmatic-serialization attribute may start while its predecessor in
// the stream is still running; grid_dep_wait() blocks until the predecessor
// has completed and its writes are visible.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void grid_dep_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void grid_dep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename Kernel, typename... Args>
cudaError_t launch_pdl(Kernel kernel, dim3 grid, dim3 block, size_t smem,
                       cudaStream_t stream, bool pdl, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

inline bool aligned16(const void *p) { return ((uintptr_t)p & 15u) == 0; }

}  // namespace li
