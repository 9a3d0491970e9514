// Host-side status plumbing shared by every entry of the C ABI.
#include "li_common.cuh"

#include <mutex>

int li_tu_status_dense(int clear);
int li_tu_status_qgemv(int clear);
int li_tu_status_deltanet(int clear);
int li_tu_status_tcgemm(int clear);
int li_tu_status_prefill(int clear);
int li_tu_status_gemm_bf16(int clear);
int li_tu_status_selftest(int clear);
int li_tu_status_attn(int clear);

namespace li {

// The reference's entries return void and report nothing
// (cuda/leaninfer-fused-deltanet.cu:331-366 has no error check); their
// replacements record the first failure per host thread here.
static thread_local int t_last_error = 0;

void set_last_error(int code) {
    if (code != 0 && t_last_error == 0) t_last_error = code;
}

int launch_status() { return (int)cudaGetLastError(); }

int num_sms() {
    static std::mutex mu;
    static int cache[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    std::lock_guard<std::mutex> lock(mu);
    if (cache[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
            n = 148;
        cache[dev] = n;
    }
    return cache[dev];
}

}  // namespace li

extern "C" {

int li_get_last_error(void) {
    const int e = li::t_last_error;
    li::t_last_error = 0;
    return e;
}

size_t li_row_bytes(int wtype, int64_t k) {
    if (k <= 0) return 0;
    switch (wtype) {
    case LI_WTYPE_F32: return (size_t)k * 4;
    case LI_WTYPE_F16: return (size_t)k * 2;
    case LI_WTYPE_Q8_0: return (k % 32) ? 0 : (size_t)(k / 32) * li::kQ80Bytes;
    case LI_WTYPE_Q4_K: return (k % 256) ? 0 : (size_t)(k / 256) * li::kQ4KBytes;
    default: return 0;
    }
}

}  // extern "C"

namespace li {
namespace {

// dst = a + b, four floats per thread when the pointers allow (the residual
// adds between the layers of a decode stack); a programmatic dependent launch.
__global__ void __launch_bounds__(256) add_f32_kernel(float *dst, const float *a, const float *b, int64_t n,
                                                      bool vec) {
    grid_dep_wait();
    grid_dep_launch_dependents();
    const int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x;
    if (vec) {
        if (4 * i + 3 < n) {
            const float4 x = reinterpret_cast<const float4 *>(a)[i], y = reinterpret_cast<const float4 *>(b)[i];
            reinterpret_cast<float4 *>(dst)[i] = make_float4(x.x + y.x, x.y + y.y, x.z + y.z, x.w + y.w);
        }
    } else if (i < n) {
        dst[i] = a[i] + b[i];
    }
}

}  // namespace
}  // namespace li

extern "C" {

int li_launch_add_f32(float *dst, const float *a, const float *b, int64_t n, void *stream) {
    if (!dst || !a || !b || n < 0) return LI_ERR_BAD_ARG;
    if (n == 0) return 0;
    const bool vec = n % 4 == 0 && li::aligned16(dst) && li::aligned16(a) && li::aligned16(b);
    const int64_t items = vec ? n / 4 : n;
    return (int)li::launch_pdl(li::add_f32_kernel, dim3((unsigned)((items + 255) / 256)), dim3(256), 0,
                               (cudaStream_t)stream, true, dst, a, b, n, vec);
}

// Synchronises the current device, then returns and clears the device-side
// failure flag raised by a bounded wait that gave up (LI_ERR_TIMEOUT), or a
// CUDA error from the synchronisation. Not for use inside graph capture.
int li_device_status(void) {
    const cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return (int)e;
    int s = 0, v;
    if ((v = li_tu_status_dense(1)) && !s) s = v;
    if ((v = li_tu_status_qgemv(1)) && !s) s = v;
    if ((v = li_tu_status_deltanet(1)) && !s) s = v;
    if ((v = li_tu_status_tcgemm(1)) && !s) s = v;
    if ((v = li_tu_status_prefill(1)) && !s) s = v;
    if ((v = li_tu_status_gemm_bf16(1)) && !s) s = v;
    if ((v = li_tu_status_selftest(1)) && !s) s = v;
    if ((v = li_tu_status_attn(1)) && !s) s = v;
    return s;
}

}  // extern "C"
