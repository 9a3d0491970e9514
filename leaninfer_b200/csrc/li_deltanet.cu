// Gated DeltaNet recurrence and the fused decode layer.
//
// Entries:
//   li_launch_fused_deltanet_recurrent_out_f32  (reference
//       cuda/leaninfer-fused-deltanet.cu:331-366, same arguments)
//   li_launch_deltanet_recurrent_f32             (recurrence only, in-place state)
//   li_launch_deltanet_layer_decode              (whole layer, one token/sequence)
//
// Recurrence kernel: one CTA per (sequence, v-head, block of RB value rows),
// 256 threads = 8 warps; RB = 128, 64 or 32 picks 1, 2 or 4 CTAs per head so
// small batches still spread over the SMs. The CTA's slice of the fp32 state
// S[D(k)][D(v)] lives in registers for all tokens: lane l owns value rows
// row0 + (RB/32)*l .. and warp w owns key columns w, w+8, ..., so every
// state load/store is a warp-wide contiguous RB*4-byte column segment, all
// issued before the first use. Per token: u = S^T k and w = S^T q~ as
// per-thread partials over the thread's columns, an 8-way cross-warp sum in
// shared memory, v' and o on RB threads, then the rank-1 update in
// registers. In layer mode the CTAs of one head form a thread-block cluster
// and combine the gated RMSNorm's sum of squares through distributed shared
// memory. Arithmetic follows the reference
// kernel (cuda/leaninfer-fused-deltanet.cu:217-288): q~ = q*D^-1/2,
// beta = sigmoid, decay = exp(min(g,50)), clamp to +-1e6.
//
// Layer decode = three stream-ordered kernels, each launched as a
// programmatic dependent so it starts while its predecessor drains:
//   1. in-projection GEMV (li_qgemv.cu) with the causal-conv1d + SiLU
//      epilogue that also shifts the conv state;
//   2. this file's recurrence in layer mode: q/k L2 norm, beta, g from the
//      projected alpha, the recurrence, and the gated RMSNorm of the head
//      (reference cuda/leaninfer-fused-gate.cu:39-85) into the workspace;
//   3. out-projection GEMV (li_qgemv.cu) of the gated heads.
// Kernel 2 reads its state before griddepcontrol.wait; this is safe because
// the GEMV kernels let their dependents launch only after their own
// griddepcontrol.wait: kernel 2 starts once kernel 1's predecessor (the
// previous step's last kernel, which itself waited for the previous
// recurrence) has completed. (The tensor-core path gets the same order from
// its x prep, which lets the GEMM after it launch only when it completes.)
#include "li_common.cuh"
#include "li_qgemv.cuh"
#include "li_tcgemm.cuh"

#include <cooperative_groups.h>
#include <mutex>

namespace cg = cooperative_groups;

LI_DEFINE_TU_STATUS(deltanet)

namespace li {
namespace {

constexpr int kRecThreads = 256;
// Three resident CTAs per SM (registers capped at 80 per thread, a few
// spilled): more state loads stay in flight while other CTAs compute.
constexpr int kRecMinBlocks = 3;
constexpr int kRecWarps = 8;

struct RecArgs {
    // reference layouts (legacy mode)
    const float *q, *k, *v, *g, *beta;
    const float *state_in;
    float *out, *state_out;
    int64_t n_tokens, n_heads, gqa, n_seqs;
    int repeat_type;
    size_t vnb1, vnb2, vnb3;
    // layer mode
    const float *proj;      // [B][NI]: act(q|k|v) | z | beta | alpha
    int NI, Hk, C;
    const float *a_log, *dt_bias, *norm_w;
    float l2_eps, norm_eps;
    float *o_gated;         // [B][Hv*D] fp32, or
    __half *o_gated16;      // [B][Hv*D] f16 (the tensor-core out-projection's operand)
    int og16_npad;          // > 0: o_gated16 tiled for the X-stationary out-projection
    float *zero_out;        // layer output to clear for a K-split out-projection, or nullptr
    int64_t zero_len;       // floats in zero_out
    // layer mode with the state stored as fp16 (same element order)
    const __half *state_in16;
    __half *state_out16;
};

template <int D>
struct RecLayout {
    static constexpr int RPL = D / 32;            // rows per lane
    static constexpr int CPW = D / kRecWarps;     // columns per warp
};

template <int RPL>
struct VecT;
template <>
struct VecT<4> { using T = float4; };
template <>
struct VecT<2> { using T = float2; };
template <>
struct VecT<1> { using T = float; };

template <int RPL>
__device__ __forceinline__ void vload(float *dst, const float *src) {
    typename VecT<RPL>::T v = *reinterpret_cast<const typename VecT<RPL>::T *>(src);
    const float *pv = reinterpret_cast<const float *>(&v);
#pragma unroll
    for (int r = 0; r < RPL; ++r) dst[r] = pv[r];
}

template <int RPL>
__device__ __forceinline__ void vstore(float *dst, const float *src) {
    typename VecT<RPL>::T v;
    float *pv = reinterpret_cast<float *>(&v);
#pragma unroll
    for (int r = 0; r < RPL; ++r) pv[r] = src[r];
    *reinterpret_cast<typename VecT<RPL>::T *>(dst) = v;
}

// The same for a state stored as fp16: one 2*RPL-byte access, fp32 in
// registers; stores saturate at the fp16 maximum.
template <int RPL>
__device__ __forceinline__ void vload_h(float *dst, const __half *src) {
    if constexpr (RPL == 4) {
        const uint2 v = *reinterpret_cast<const uint2 *>(src);
        const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&v.x));
        const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&v.y));
        dst[0] = a.x; dst[1] = a.y; dst[2] = b.x; dst[3] = b.y;
    } else if constexpr (RPL == 2) {
        const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(src));
        dst[0] = a.x; dst[1] = a.y;
    } else {
        dst[0] = __half2float(*src);
    }
}

template <int RPL>
__device__ __forceinline__ void vstore_h(__half *dst, const float *src) {
    float c[RPL];
#pragma unroll
    for (int r = 0; r < RPL; ++r) c[r] = fminf(fmaxf(src[r], -65504.0f), 65504.0f);
    if constexpr (RPL == 4) {
        const __half2 a = __floats2half2_rn(c[0], c[1]), b = __floats2half2_rn(c[2], c[3]);
        uint2 v;
        v.x = *reinterpret_cast<const uint32_t *>(&a);
        v.y = *reinterpret_cast<const uint32_t *>(&b);
        *reinterpret_cast<uint2 *>(dst) = v;
    } else if constexpr (RPL == 2) {
        *reinterpret_cast<__half2 *>(dst) = __floats2half2_rn(c[0], c[1]);
    } else {
        *dst = __float2half_rn(c[0]);
    }
}

// SH: the state is stored as fp16 (layer mode only).
template <int D, bool LAYER, int RB, bool SH = false>
__global__ void __launch_bounds__(kRecThreads, kRecMinBlocks)
recurrent_kernel(RecArgs a) {
    constexpr int RPL = RB / 32;                 // value rows per lane
    constexpr int CPW = D / kRecWarps;           // key columns per warp
    constexpr int CS = D / RB;                   // CTAs per head
    __shared__ __align__(16) float s_q[D];
    __shared__ __align__(16) float s_k[D];
    __shared__ __align__(16) float s_vp[RB];
    __shared__ __align__(16) float s_red[kRecWarps][2][RB];
    __shared__ float s_scal[8];
    __shared__ float s_part;                     // this CTA's sum of o^2 (cluster-visible)

    const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
    const int rank = CS == 1 ? 0 : (int)(blockIdx.x % CS);
    const int64_t hblk = blockIdx.x / CS;
    const int64_t seq = hblk / a.n_heads;
    const int64_t h = hblk % a.n_heads;
    const int64_t nkq = a.n_heads / a.gqa;
    const int64_t hk = a.repeat_type == 0 ? h / a.gqa : h % nkq;   // ref :165-167
    const int row0 = rank * RB;
    const float scale = rsqrtf((float)D);

    // ---- state slice -> registers (independent of the previous kernel) ----
    float S[CPW][RPL];
    if constexpr (SH) {
        const __half *Sin = a.state_in16 + ((size_t)seq * a.n_heads + h) * D * D + row0;
#pragma unroll
        for (int j = 0; j < CPW; ++j) vload_h<RPL>(S[j], Sin + (size_t)(warp + kRecWarps * j) * D + RPL * lane);
    } else {
        const float *Sin = a.state_in + ((size_t)seq * a.n_heads + h) * D * D + row0;
#pragma unroll
        for (int j = 0; j < CPW; ++j) vload<RPL>(S[j], Sin + (size_t)(warp + kRecWarps * j) * D + RPL * lane);
    }

    if (LAYER) {
        grid_dep_launch_dependents();
        grid_dep_wait();
        if (a.zero_out) {
            // the out-projection that follows adds K-split partials into it
            const int64_t per = (a.zero_len + gridDim.x - 1) / gridDim.x;
            const int64_t z0 = (int64_t)blockIdx.x * per;
            const int64_t z1 = z0 + per < a.zero_len ? z0 + per : a.zero_len;
            for (int64_t i = z0 + threadIdx.x; i < z1; i += blockDim.x) a.zero_out[i] = 0.f;
        }
    }
    // Layer mode (one token): this thread's projected v and z are loaded now,
    // next to q and k, so the token's phases wait for no further global load.
    float v_pre = 0.f, z_pre = 0.f;
    if (LAYER && threadIdx.x < RB) {
        const float *pr = a.proj + (size_t)seq * a.NI + h * D + row0 + threadIdx.x;
        v_pre = pr[2 * a.Hk * D];
        z_pre = pr[a.C];
    }

    for (int64_t t = 0; t < a.n_tokens; ++t) {
        float beta_s, decay;
        if (!LAYER) {
            const float *qp = a.q + ((seq * nkq + hk) * a.n_tokens + t) * D;
            const float *kp = a.k + ((seq * nkq + hk) * a.n_tokens + t) * D;
            for (int i = threadIdx.x; i < D; i += kRecThreads) {
                s_q[i] = qp[i] * scale;
                s_k[i] = kp[i];
            }
            const float gb = a.g[(seq * a.n_tokens + t) * a.n_heads + h];
            const float bb = a.beta[(seq * a.n_tokens + t) * a.n_heads + h];
            beta_s = 1.0f / (1.0f + expf(-bb));
            decay = expf(fminf(gb, 50.0f));
        } else {
            const float *pr = a.proj + (size_t)seq * a.NI;
            const int Hv = (int)a.n_heads;
            // q, k of k-head hk, L2-normalised (warp 0: q, warp 1: k)
            if (warp < 2) {
                constexpr int E = D / 32;
                const float *src = pr + (warp == 0 ? 0 : a.Hk * D) + hk * D;
                float vals[E];
                float sq = 0.f;
#pragma unroll
                for (int r = 0; r < E; ++r) {
                    vals[r] = src[E * lane + r];
                    sq = fmaf(vals[r], vals[r], sq);
                }
                const float inv = rsqrtf(warp_sum(sq) + a.l2_eps);
                float *dst = warp == 0 ? s_q : s_k;
                const float f = warp == 0 ? inv * scale : inv;
#pragma unroll
                for (int r = 0; r < E; ++r) dst[E * lane + r] = vals[r] * f;
            }
            const float braw = pr[a.C + Hv * D + h];
            const float araw = pr[a.C + Hv * D + Hv + h];
            beta_s = sigmoid(braw);
            const float gval = -expf(a.a_log[h]) * softplus(araw + a.dt_bias[h]);
            decay = expf(fminf(gval, 50.0f));
        }
        __syncthreads();

        // k . q~ (every warp computes it; no extra barrier)
        float kq = 0.f;
#pragma unroll
        for (int i = 0; i < D / kWarp; ++i) kq = fmaf(s_k[lane + kWarp * i], s_q[lane + kWarp * i], kq);
        const float attn = warp_sum(kq);

        // partial u = S^T k, w = S^T q~ over this thread's columns
        float pu[RPL], pw[RPL];
#pragma unroll
        for (int r = 0; r < RPL; ++r) pu[r] = pw[r] = 0.f;
#pragma unroll
        for (int j = 0; j < CPW; ++j) {
            const int c = warp + kRecWarps * j;
            const float kc = s_k[c], qc = s_q[c];
#pragma unroll
            for (int r = 0; r < RPL; ++r) {
                pu[r] = fmaf(S[j][r], kc, pu[r]);
                pw[r] = fmaf(S[j][r], qc, pw[r]);
            }
        }
        vstore<RPL>(&s_red[warp][0][RPL * lane], pu);
        vstore<RPL>(&s_red[warp][1][RPL * lane], pw);
        __syncthreads();

        float o = 0.f;
        if (threadIdx.x < RB) {
            const int r = threadIdx.x;
            float u = 0.f, w = 0.f;
#pragma unroll
            for (int ww = 0; ww < kRecWarps; ++ww) {
                u += s_red[ww][0][r];
                w += s_red[ww][1][r];
            }
            float vv;
            if (!LAYER)
                vv = a.v[seq * a.vnb3 + h * a.vnb2 + t * a.vnb1 + row0 + r];
            else
                vv = v_pre;
            const float vn = beta_s * (vv - u * decay);
            o = w * decay + vn * attn;
            s_vp[r] = vn;
            if (!LAYER) {
                a.out[((seq * a.n_tokens + t) * a.n_heads + h) * D + row0 + r] = o;
            } else {
                const float sq = warp_sum(o * o);
                if ((r % kWarp) == 0) s_scal[r / kWarp] = sq;
            }
        }
        __syncthreads();
        if (LAYER) {
            // gated RMSNorm of the head (reference cuda/leaninfer-fused-gate.cu:39-85):
            // sum o^2 over the CS CTAs of the cluster
            if (threadIdx.x == 0) {
                float p = 0.f;
#pragma unroll
                for (int i = 0; i < RB / kWarp; ++i) p += s_scal[i];
                s_part = p;
            }
            float tot;
            if (CS == 1) {
                __syncthreads();
                tot = s_part;
            } else {
                cg::cluster_group cluster = cg::this_cluster();
                cluster.sync();
                tot = 0.f;
#pragma unroll
                for (int i = 0; i < CS; ++i) tot += *cluster.map_shared_rank(&s_part, i);
            }
            if (threadIdx.x < RB) {
                const int r = threadIdx.x;
                const float rs = rsqrtf(tot / (float)D + a.norm_eps);
                const float z = z_pre;
                const float og = silu(z) * (o * a.norm_w[row0 + r] * rs);
                const size_t oi = ((size_t)seq * a.n_heads + h) * D + row0 + r;
                if (a.o_gated16)
                    a.o_gated16[a.og16_npad ? tiled_x_offset(seq, h * D + row0 + r, a.og16_npad) : oi] =
                        __float2half_rn(og);
                else a.o_gated[oi] = og;
            }
        }

        // S <- clamp(decay*S + k v'^T)
        float vp[RPL];
        vload<RPL>(vp, &s_vp[RPL * lane]);
#pragma unroll
        for (int j = 0; j < CPW; ++j) {
            const float kc = s_k[warp + kRecWarps * j];
#pragma unroll
            for (int r = 0; r < RPL; ++r)
                S[j][r] = fminf(fmaxf(fmaf(decay, S[j][r], vp[r] * kc), -1e6f), 1e6f);
        }
        __syncthreads();   // s_q/s_k/s_vp/s_red reused by the next token
    }

    if constexpr (SH) {
        __half *Sout = a.state_out16 + ((size_t)seq * a.n_heads + h) * D * D + row0;
#pragma unroll
        for (int j = 0; j < CPW; ++j) vstore_h<RPL>(Sout + (size_t)(warp + kRecWarps * j) * D + RPL * lane, S[j]);
    } else {
        float *Sout = a.state_out + ((size_t)seq * a.n_heads + h) * D * D + row0;
#pragma unroll
        for (int j = 0; j < CPW; ++j) vstore<RPL>(Sout + (size_t)(warp + kRecWarps * j) * D + RPL * lane, S[j]);
    }
    if (LAYER && CS > 1) {
        // No CTA leaves while a cluster peer may still read its s_part. Only
        // shared-memory lifetime is at stake, so the arrive is relaxed: it
        // does not wait for this thread's global stores to become visible.
        asm volatile("barrier.cluster.arrive.relaxed.aligned;\n\tbarrier.cluster.wait.aligned;" ::: "memory");
    }
}

// proj[d][t] = sum_s sum_j W[d][j] * o[s][t][j], o [n_seqs][n_tok][HD]
// (the reference's intended out-projection, cuda/leaninfer-fused-deltanet.cu:260-279).
__global__ void __launch_bounds__(256)
proj_f32_kernel(const float *__restrict__ W, const float *__restrict__ o, float *__restrict__ proj,
                int64_t hidden, int64_t n_tok, int64_t n_seqs, int64_t HD) {
    const int64_t d = (int64_t)blockIdx.x * 8 + threadIdx.x / kWarp;
    const int lane = threadIdx.x % kWarp;
    if (d >= hidden) return;
    const float *wr = W + d * HD;
    for (int64_t t = 0; t < n_tok; ++t) {
        float acc = 0.f;
        for (int64_t j = lane; j < HD; j += kWarp) {
            float os = 0.f;
            for (int64_t s = 0; s < n_seqs; ++s) os += o[(s * n_tok + t) * HD + j];
            acc = fmaf(wr[j], os, acc);
        }
        acc = warp_sum(acc);
        if (lane == 0) proj[d * n_tok + t] = acc;
    }
}

int check_rec(const float *q, const float *k, const float *v, const float *g, const float *beta,
              const float *state_in, int64_t head_dim, int64_t n_tokens, int64_t n_heads,
              int64_t gqa, int64_t n_seqs) {
    if (!q || !k || !v || !g || !beta || !state_in) return LI_ERR_BAD_ARG;
    if (n_tokens < 0 || n_heads <= 0 || gqa <= 0 || n_seqs < 0) return LI_ERR_BAD_ARG;
    if (n_heads % gqa) return LI_ERR_BAD_SHAPE;
    if (head_dim != 128 && head_dim != 64) return LI_ERR_UNSUPPORTED;
    if (n_seqs * n_heads > 0x7fffffffLL) return LI_ERR_BAD_SHAPE;
    return 0;
}

// Value rows per CTA: enough CTAs to cover the SMs at small batch.
int pick_rows(int64_t heads_total, int64_t head_dim) {
    if (head_dim == 64) return heads_total <= 128 ? 32 : 64;
    return heads_total <= 64 ? 32 : (heads_total <= 512 ? 64 : 128);
}

int launch_rec(const RecArgs &a, int64_t head_dim, cudaStream_t stream) {
    const int64_t heads = a.n_seqs * a.n_heads;
    if (heads == 0) return 0;
    const int rb = pick_rows(heads, head_dim);
    const unsigned grid = (unsigned)(heads * (head_dim / rb));
    if (head_dim == 128) {
        if (rb == 32) recurrent_kernel<128, false, 32><<<grid, kRecThreads, 0, stream>>>(a);
        else if (rb == 64) recurrent_kernel<128, false, 64><<<grid, kRecThreads, 0, stream>>>(a);
        else recurrent_kernel<128, false, 128><<<grid, kRecThreads, 0, stream>>>(a);
    } else {
        if (rb == 32) recurrent_kernel<64, false, 32><<<grid, kRecThreads, 0, stream>>>(a);
        else recurrent_kernel<64, false, 64><<<grid, kRecThreads, 0, stream>>>(a);
    }
    return launch_status();
}

// Layer-mode launch: a cluster of D/RB CTAs per head, programmatic dependent.
template <int RB, bool SH = false>
int launch_layer_rec(const RecArgs &a, cudaStream_t stream) {
    const int64_t heads = a.n_seqs * a.n_heads;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(heads * (128 / RB)));
    cfg.blockDim = dim3(kRecThreads);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 128 / RB;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return (int)cudaLaunchKernelEx(&cfg, recurrent_kernel<128, true, RB, SH>, a);
}

int launch_layer_rec_any(const RecArgs &a, int rb, bool sh, cudaStream_t s) {
    if (sh) return rb == 32 ? launch_layer_rec<32, true>(a, s) : rb == 64 ? launch_layer_rec<64, true>(a, s)
                                                                       : launch_layer_rec<128, true>(a, s);
    return rb == 32 ? launch_layer_rec<32>(a, s) : rb == 64 ? launch_layer_rec<64>(a, s) : launch_layer_rec<128>(a, s);
}

}  // namespace
}  // namespace li

using namespace li;

extern "C" {

int li_launch_deltanet_recurrent_f32(const float *q, const float *k, const float *v,
                                     const float *g, const float *beta, const float *state_in,
                                     float *out, float *state_out, int64_t head_dim,
                                     int64_t n_tokens, int64_t n_heads, int64_t gqa_ratio,
                                     int repeat_type, int64_t n_seqs, size_t vnb1, size_t vnb2,
                                     size_t vnb3, void *stream) {
    int rc = check_rec(q, k, v, g, beta, state_in, head_dim, n_tokens, n_heads, gqa_ratio, n_seqs);
    if (rc) return rc;
    if (!out || !state_out) return LI_ERR_BAD_ARG;
    if (!aligned16(state_in) || !aligned16(state_out)) return LI_ERR_MISALIGNED;
    RecArgs a = {};
    a.q = q; a.k = k; a.v = v; a.g = g; a.beta = beta;
    a.state_in = state_in; a.out = out; a.state_out = state_out;
    a.n_tokens = n_tokens; a.n_heads = n_heads; a.gqa = gqa_ratio; a.n_seqs = n_seqs;
    a.repeat_type = repeat_type; a.vnb1 = vnb1; a.vnb2 = vnb2; a.vnb3 = vnb3;
    return launch_rec(a, head_dim, (cudaStream_t)stream);
}

void li_launch_fused_deltanet_recurrent_out_f32(const float *q, const float *k, const float *v,
                                                const float *g, const float *beta,
                                                const float *state_in, const float *W_out,
                                                float *dst, float *proj_out, int64_t head_dim,
                                                int64_t n_tokens, int64_t n_heads,
                                                int64_t gqa_ratio, int repeat_type, int64_t n_seqs,
                                                int64_t hidden_dim, size_t vnb1, size_t vnb2,
                                                size_t vnb3, void *stream) {
    int rc = check_rec(q, k, v, g, beta, state_in, head_dim, n_tokens, n_heads, gqa_ratio, n_seqs);
    if (!rc && !dst) rc = LI_ERR_BAD_ARG;
    if (!rc && (!aligned16(state_in) || !aligned16(dst))) rc = LI_ERR_MISALIGNED;
    const cudaStream_t s = (cudaStream_t)stream;
    const int64_t out_elems = head_dim * n_tokens * n_heads * n_seqs;   // ref :342
    if (!rc && (out_elems * 4) % 16) rc = LI_ERR_MISALIGNED;           // state after outputs
    if (!rc) {
        RecArgs a = {};
        a.q = q; a.k = k; a.v = v; a.g = g; a.beta = beta;
        a.state_in = state_in; a.out = dst; a.state_out = dst + out_elems;
        a.n_tokens = n_tokens; a.n_heads = n_heads; a.gqa = gqa_ratio; a.n_seqs = n_seqs;
        a.repeat_type = repeat_type; a.vnb1 = vnb1; a.vnb2 = vnb2; a.vnb3 = vnb3;
        rc = launch_rec(a, head_dim, s);
    }
    if (!rc && proj_out && W_out && hidden_dim > 0 && n_tokens > 0) {
        const unsigned grid = (unsigned)((hidden_dim + 7) / 8);
        proj_f32_kernel<<<grid, 256, 0, s>>>(W_out, dst, proj_out, hidden_dim, n_tokens, n_seqs,
                                             n_heads * head_dim);
        rc = launch_status();
    }
    set_last_error(rc);
}

// Workspace regions, each 256-byte aligned:
//   SIMT path:   proj f32 [B][NI] | og f32 [B][Hv*D]
//   tensor path: proj f32 [B][NI] | x16 f16 [B][hidden] | xscale f32 [B] |
//                og16 f16 [B][Hv*D] | partial sums
static size_t al256(size_t v) { return (v + 255) / 256 * 256; }

// The projections run on the SIMT GEMV kernels below kTcMinRows sequences,
// and up to kLayerFewRowsMax when both projection shapes suit the few-row
// kernel (weights read once into registers, no f16 operand and no partial
// sums); on the tensor cores otherwise. Measured on B200 at hidden 4096,
// Q4_K, layer step: 2 sequences 30 us (staged SIMT 44), 3: 37.5 (tensor
// cores 43), 4: 44 either way, 6: 63 (tensor cores 46; the few-row kernel
// reads every x row from shared memory once per weight row pair). Decided
// from shapes alone, so the workspace size and the launch agree.
constexpr int kLayerFewRowsMax = 3;
static bool layer_simt(const li_deltanet_layer *L, int n_seqs) {
    if (n_seqs < li::kTcMinRows) return true;
    return n_seqs <= kLayerFewRowsMax && li::qgemv_few_rows(L->w_in_type, L->hidden, n_seqs) &&
           li::qgemv_few_rows(L->w_out_type, L->n_v_heads * L->head_dim, n_seqs);
}

// partial sums of the X-stationary projections (the in- and out-projection
// run one after the other and share the region)
static size_t layer_partials_bytes(const li_deltanet_layer *L, int n_seqs) {
    const int D = L->head_dim, Hk = L->n_k_heads, Hv = L->n_v_heads;
    const int NI = 2 * Hk * D + 2 * Hv * D + 2 * Hv;
    const size_t pin = li::tc_gemm_partials_bytes(L->w_in_type, li::kTcConv, L->hidden, NI, n_seqs);
    const size_t pout = li::tc_gemm_partials_bytes(L->w_out_type, li::kTcStore, Hv * D, L->hidden, n_seqs);
    return pin > pout ? pin : pout;
}

size_t li_deltanet_layer_workspace_size(const li_deltanet_layer *L, int n_seqs) {
    if (!L || n_seqs <= 0) return 0;
    const size_t D = L->head_dim, Hk = L->n_k_heads, Hv = L->n_v_heads, n = (size_t)n_seqs;
    const size_t NI = 2 * Hk * D + 2 * Hv * D + 2 * Hv;
    if (layer_simt(L, n_seqs)) return al256(NI * n * 4) + al256(Hv * D * n * 4);
    const size_t nx = (n + 31) / 32 * 32;   // tiled X operands are padded to 32 rows
    return al256(NI * n * 4) + al256((size_t)L->hidden * nx * 2) + al256(n * 4) + al256(Hv * D * nx * 2) +
           al256(layer_partials_bytes(L, n_seqs));
}

}  // extern "C"

// The layer step; the state is fp32 (`state`) or fp16 (`state16`).
// accumulate: y += the layer's output (the out-projection adds into y).
static int layer_decode(const li_deltanet_layer *L, const float *x, float *y, float *conv_state, float *state,
                        __half *state16, int n_seqs, void *workspace, size_t workspace_bytes, void *stream,
                        bool accumulate = false) {
    if (!L || !x || !y || !conv_state || (!state && !state16) || n_seqs < 0) return LI_ERR_BAD_ARG;
    if (!state) state = reinterpret_cast<float *>(state16);   // alignment check below covers both
    if (n_seqs == 0) return 0;
    if (!L->w_in || !L->conv_w || !L->a_log || !L->dt_bias || !L->norm_w || !L->w_out)
        return LI_ERR_BAD_ARG;
    if (L->head_dim != 128 || L->conv_kernel != 4) return LI_ERR_UNSUPPORTED;
    if (L->n_k_heads <= 0 || L->n_v_heads <= 0 || L->n_v_heads % L->n_k_heads) return LI_ERR_BAD_SHAPE;
    if (!aligned16(state) || !aligned16(L->conv_w) || !aligned16(x)) return LI_ERR_MISALIGNED;
    if (L->in_norm_w && !aligned16(L->in_norm_w)) return LI_ERR_MISALIGNED;
    if (!workspace || workspace_bytes < li_deltanet_layer_workspace_size(L, n_seqs))
        return LI_ERR_WORKSPACE;
    const int D = L->head_dim, Hk = L->n_k_heads, Hv = L->n_v_heads;
    const int C = 2 * Hk * D + Hv * D;
    const int NI = C + Hv * D + 2 * Hv;
    const size_t n = (size_t)n_seqs;
    char *ws = (char *)workspace;
    float *proj = (float *)ws;
    const cudaStream_t s = (cudaStream_t)stream;
    const bool tc = !layer_simt(L, n_seqs);
    int rc;

    RecArgs a = {};
    a.state_in = state16 ? nullptr : state; a.state_out = state16 ? nullptr : state;
    a.state_in16 = state16; a.state_out16 = state16;
    a.n_tokens = 1; a.n_heads = Hv; a.gqa = Hv / Hk; a.n_seqs = n_seqs;
    a.repeat_type = L->repeat_type;
    a.proj = proj; a.NI = NI; a.Hk = Hk; a.C = C;
    a.a_log = L->a_log; a.dt_bias = L->dt_bias; a.norm_w = L->norm_w;
    a.l2_eps = L->l2_eps; a.norm_eps = L->norm_eps;
    const int rb = pick_rows((int64_t)n_seqs * Hv, 128);

    if (!tc) {
        float *og = (float *)(ws + al256((size_t)NI * n * 4));
        // 1. in-projection + conv1d/SiLU epilogue (dependent launch: weights
        //    and the conv state are read before its wait, x after it)
        QGemvArgs in = {};
        in.wtype = L->w_in_type; in.epi = kEpiConv;
        if ((rc = qgemv_plan(L->w_in_type, L->hidden, NI, kEpiConv, &in.plan))) return rc;
        in.x = x; in.x_stride = L->hidden; in.gamma = L->in_norm_w; in.K = L->hidden;
        in.eps = L->in_norm_eps; in.n_seg = 1; in.W[0] = L->w_in; in.seg_rows[0] = NI;
        in.dst[0] = proj; in.dst_stride[0] = NI;
        in.conv_w = L->conv_w; in.conv_state = conv_state; in.conv_channels = C;
        if ((rc = qgemv_launch(in, n_seqs, s, true))) return rc;
        // 2. recurrence + L2 norm + gated RMSNorm (dependent launch)
        a.o_gated = og;
        rc = launch_layer_rec_any(a, rb, state16 != nullptr, s);
        if (rc) return rc;
        // 3. out-projection (dependent launch)
        QGemvArgs out = {};
        out.wtype = L->w_out_type; out.epi = kEpiStore;
        if ((rc = qgemv_plan(L->w_out_type, Hv * D, L->hidden, kEpiStore, &out.plan))) return rc;
        out.x = og; out.x_stride = Hv * D; out.gamma = nullptr; out.K = Hv * D; out.eps = 0.f;
        out.n_seg = 1; out.W[0] = L->w_out; out.seg_rows[0] = L->hidden;
        out.dst[0] = y; out.dst_stride[0] = L->hidden;
        out.accumulate = accumulate;
        return qgemv_launch(out, n_seqs, s, true);
    }

    // tensor-core path: x -> f16, in-projection GEMM (+conv), recurrence
    // (gated heads written as f16), out-projection GEMM
    const size_t nx = (n + 31) / 32 * 32;
    size_t off = al256((size_t)NI * n * 4);
    __half *x16 = (__half *)(ws + off);
    off += al256((size_t)L->hidden * nx * 2);
    float *xscale = (float *)(ws + off);
    off += al256(n * 4);
    __half *og16 = (__half *)(ws + off);
    off += al256(Hv * D * nx * 2);
    float *partials = layer_partials_bytes(L, n_seqs) ? (float *)(ws + off) : nullptr;
    TcArgs in = {};
    in.wtype = L->w_in_type; in.epi = kTcConv; in.K = L->hidden; in.total_rows = NI; in.B = n_seqs;
    in.W[0] = L->w_in; in.n_seg = 1; in.seg_rows[0] = NI; in.dst[0] = proj; in.dst_stride[0] = NI;
    in.X16 = x16; in.xscale = xscale;
    in.conv_w = L->conv_w; in.conv_state = conv_state; in.conv_channels = C;
    in.partials = partials;
    in.x_npad = tc_gemm_x_npad(in);
    if (tc_gemm_splits_k(in)) {
        // the K-split in-projection adds its partial sums into proj (the conv
        // epilogue follows in its own kernel)
        const cudaError_t e = cudaMemsetAsync(proj, 0, (size_t)NI * n * sizeof(float), s);
        if (e != cudaSuccess) return (int)e;
    }
    // a dependent launch: the prep waits for the previous kernel before it reads x
    if ((rc = tc_prep_launch(x, L->hidden, L->in_norm_w, L->in_norm_eps, n_seqs, L->hidden, x16, xscale, s,
                             true, in.x_npad, tc_gemm_x_stationary(in))))
        return rc;
    if ((rc = tc_gemm_launch(in, s, true))) return rc;
    TcArgs out = {};
    out.wtype = L->w_out_type; out.epi = kTcStore; out.K = Hv * D; out.total_rows = L->hidden; out.B = n_seqs;
    out.W[0] = L->w_out; out.n_seg = 1; out.seg_rows[0] = L->hidden; out.dst[0] = y;
    out.dst_stride[0] = L->hidden; out.X16 = og16; out.xscale = nullptr;
    out.partials = partials;
    out.accumulate = accumulate;
    out.x_npad = tc_gemm_x_npad(out);
    a.o_gated16 = og16;
    a.og16_npad = out.x_npad;
    if (tc_gemm_splits_k(out) && !accumulate) {
        a.zero_out = y;
        a.zero_len = (int64_t)n_seqs * L->hidden;
    }
    rc = launch_layer_rec_any(a, rb, state16 != nullptr, s);
    if (rc) return rc;
    return tc_gemm_launch(out, s, true);
}

extern "C" {

int li_launch_deltanet_layer_decode(const li_deltanet_layer *L, const float *x, float *y,
                                    float *conv_state, float *state, int n_seqs, void *workspace,
                                    size_t workspace_bytes, void *stream) {
    if (!state) return LI_ERR_BAD_ARG;
    return layer_decode(L, x, y, conv_state, state, nullptr, n_seqs, workspace, workspace_bytes, stream);
}

int li_launch_deltanet_layer_decode_f16state(const li_deltanet_layer *L, const float *x, float *y,
                                             float *conv_state, void *state, int n_seqs, void *workspace,
                                             size_t workspace_bytes, void *stream) {
    if (!state) return LI_ERR_BAD_ARG;
    return layer_decode(L, x, y, conv_state, nullptr, static_cast<__half *>(state), n_seqs, workspace,
                        workspace_bytes, stream);
}

}  // extern "C"

int li::deltanet_layer_decode_residual(const li_deltanet_layer *L, const float *x, float *y, float *conv_state,
                                       float *state, int n_seqs, void *workspace, size_t workspace_bytes,
                                       void *stream) {
    if (!state) return LI_ERR_BAD_ARG;
    return layer_decode(L, x, y, conv_state, state, nullptr, n_seqs, workspace, workspace_bytes, stream, true);
}

// ---------------------------------------------------------------------------
// Layer decode with scratch in this library's own device memory.
//
// Some callers cannot hand the layer a workspace: a ggml graph whose buffers
// the graph allocator planned before this op existed, a host runtime that
// owns all device memory and passes a plugin only tensors and a stream, or a
// decode loop where an allocation call (which waits for the device) is not
// acceptable. For them the scratch is a file-scope device array of
// LI_DELTANET_STATIC_SCRATCH_BYTES, which every GPU that loads the library
// holds until the process exits. Host code cannot use the array's name as a
// device address, so its address is looked up with cudaGetSymbolAddress once
// per device, with that device current, on the first call made on it.
// ---------------------------------------------------------------------------
static __device__ __align__(256) unsigned char g_layer_scratch[LI_DELTANET_STATIC_SCRATCH_BYTES];

static int layer_scratch_address(void **out) {
    static std::mutex mu;
    static void *addr[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    if (dev < 0 || dev >= 64) return LI_ERR_UNSUPPORTED;
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[dev]) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_layer_scratch);
        if (e != cudaSuccess) return (int)e;
        addr[dev] = p;
    }
    *out = addr[dev];
    return 0;
}

extern "C" int li_launch_deltanet_layer_decode_noalloc(const li_deltanet_layer *L, const float *x,
                                                       float *y, float *conv_state, float *state,
                                                       int n_seqs, void *stream) {
    if (!L || n_seqs < 0) return LI_ERR_BAD_ARG;
    if (n_seqs == 0) return 0;
    // Every byte of the scratch that a launch reads is written earlier in the
    // same launch, so nothing has to start at zero; the array keeps the last
    // call's contents.
    if (li_deltanet_layer_workspace_size(L, n_seqs) > (size_t)LI_DELTANET_STATIC_SCRATCH_BYTES)
        return LI_ERR_SCRATCH_LIMIT;
    void *ws = nullptr;
    const int rc = layer_scratch_address(&ws);
    if (rc) return rc;
    return li_launch_deltanet_layer_decode(L, x, y, conv_state, state, n_seqs, ws,
                                           (size_t)LI_DELTANET_STATIC_SCRATCH_BYTES, stream);
}
