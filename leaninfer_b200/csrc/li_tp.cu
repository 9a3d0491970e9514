// Two-dimensional sharding of the SwiGLU FFN over NCCL (host C++ behind the
// C ABI): sequences stay sharded by rank for the mixer layers, the FFN's
// inner dimension N is split into block-aligned ranges, one per rank (W_gate
// and W_up rows column-parallel, the matching column range of every W_down
// row row-parallel). One step on rank r, R sequences per rank:
//
//   x_all  = all_gather(x)                      [nranks*R, K]  (ncclAllGather)
//   y_part = W_down_r . swiglu(rmsnorm(x_all); W_gate_r, W_up_r)
//                                               [nranks*R, K]  partial sums over N_r
//   y      = reduce_scatter(y_part, sum)         [R, K]        (ncclReduceScatter)
//
// The local products are li_launch_fused_ffn_q on the gathered rows (tensor
// cores from kTcMinRows rows). The collectives are NCCL's, issued on the
// caller's stream; nothing here waits on the host. The reference has no
// multi-GPU code: this is the 2-D scheme that lets a weight-heavy decode stack
// scale past sequence sharding (per-GPU weight bytes fall as 1/nranks).
//
// NCCL is loaded at first use with dlopen("libnccl.so.2"): the copy already
// in the process (for example PyTorch's) when there is one, so a communicator
// made by that copy can be passed in; otherwise the system's.
#include "li_common.cuh"

#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>

namespace li {
namespace {

struct NcclApi {
    ncclResult_t (*get_unique_id)(ncclUniqueId *);
    ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int);
    ncclResult_t (*comm_destroy)(ncclComm_t);
    ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*reduce_scatter)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                                   cudaStream_t);
    ncclResult_t (*comm_count)(const ncclComm_t, int *);
    bool ok;
};

const NcclApi &nccl() {
    static NcclApi api = {};
    static std::once_flag once;
    std::call_once(once, [] {
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
        api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
        api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
        api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
        api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(h, "ncclAllGather"));
        api.reduce_scatter = reinterpret_cast<decltype(api.reduce_scatter)>(dlsym(h, "ncclReduceScatter"));
        api.comm_count = reinterpret_cast<decltype(api.comm_count)>(dlsym(h, "ncclCommCount"));
        api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.all_gather &&
                 api.reduce_scatter && api.comm_count;
    });
    return api;
}

int nccl_status(ncclResult_t r) { return r == ncclSuccess ? 0 : LI_ERR_NCCL; }

size_t al256(size_t v) { return (v + 255) / 256 * 256; }

}  // namespace
}  // namespace li

using namespace li;

extern "C" {

int li_nccl_available(void) { return nccl().ok ? 1 : 0; }

int li_nccl_get_unique_id(void *id) {
    if (!id) return LI_ERR_BAD_ARG;
    if (!nccl().ok) return LI_ERR_UNSUPPORTED;
    ncclUniqueId u;
    const int rc = nccl_status(nccl().get_unique_id(&u));
    if (!rc) memcpy(id, &u, sizeof(u));
    return rc;
}

int li_nccl_comm_init_rank(void **comm, int nranks, const void *id, int rank) {
    if (!comm || !id || nranks <= 0 || rank < 0 || rank >= nranks) return LI_ERR_BAD_ARG;
    if (!nccl().ok) return LI_ERR_UNSUPPORTED;
    ncclUniqueId u;
    memcpy(&u, id, sizeof(u));
    ncclComm_t c = nullptr;
    const int rc = nccl_status(nccl().comm_init_rank(&c, nranks, u, rank));
    *comm = rc ? nullptr : (void *)c;
    return rc;
}

int li_nccl_comm_destroy(void *comm) {
    if (!comm) return LI_ERR_BAD_ARG;
    if (!nccl().ok) return LI_ERR_UNSUPPORTED;
    return nccl_status(nccl().comm_destroy((ncclComm_t)comm));
}

size_t li_ffn_tp_workspace_size(int K, int N_local, int rows_per_rank, int nranks) {
    if (K <= 0 || N_local <= 0 || rows_per_rank <= 0 || nranks <= 0) return 0;
    const size_t rows = (size_t)rows_per_rank * nranks;
    const size_t ffn = li_fused_ffn_workspace_size(K, N_local, (int)rows);
    if (nranks == 1) return ffn;
    return al256(rows * K * 4) * 2 + ffn;
}

int li_launch_ffn_q_tp(int wtype, const float *x, const float *gamma, const void *Wg, const void *Wu,
                       const void *Wd, float *y, int K, int N_local, int rows_per_rank, float eps, void *comm,
                       int nranks, void *workspace, size_t workspace_bytes, void *stream) {
    if (!x || !y || !Wg || !Wu || !Wd || K <= 0 || N_local <= 0 || rows_per_rank < 0 || nranks <= 0)
        return LI_ERR_BAD_ARG;
    if (rows_per_rank == 0) return 0;
    if ((size_t)rows_per_rank * nranks > (size_t)1 << 30) return LI_ERR_BAD_SHAPE;
    if (!workspace || workspace_bytes < li_ffn_tp_workspace_size(K, N_local, rows_per_rank, nranks))
        return LI_ERR_WORKSPACE;
    if (!aligned16(workspace)) return LI_ERR_MISALIGNED;
    const cudaStream_t s = (cudaStream_t)stream;
    const int rows = rows_per_rank * nranks;
    if (nranks == 1)
        return li_launch_fused_ffn_q(wtype, x, gamma, Wg, Wu, Wd, y, K, N_local, rows, eps, workspace,
                                     workspace_bytes, stream);
    if (!comm) return LI_ERR_BAD_ARG;
    if (!nccl().ok) return LI_ERR_UNSUPPORTED;
    int count = 0;
    if (nccl().comm_count((ncclComm_t)comm, &count) != ncclSuccess || count != nranks) return LI_ERR_BAD_ARG;
    char *ws = (char *)workspace;
    float *x_all = reinterpret_cast<float *>(ws);
    float *y_part = reinterpret_cast<float *>(ws + al256((size_t)rows * K * 4));
    char *ffn_ws = ws + 2 * al256((size_t)rows * K * 4);
    const size_t ffn_bytes = workspace_bytes - 2 * al256((size_t)rows * K * 4);
    const size_t per = (size_t)rows_per_rank * K;
    int rc = nccl_status(nccl().all_gather(x, x_all, per, ncclFloat32, (ncclComm_t)comm, s));
    if (rc) return rc;
    rc = li_launch_fused_ffn_q(wtype, x_all, gamma, Wg, Wu, Wd, y_part, K, N_local, rows, eps, ffn_ws, ffn_bytes,
                               stream);
    if (rc) return rc;
    return nccl_status(nccl().reduce_scatter(y_part, y, per, ncclFloat32, ncclSum, (ncclComm_t)comm, s));
}

}  // extern "C"
