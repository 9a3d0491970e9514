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
