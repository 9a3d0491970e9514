// Quantized (Q8_0 / Q4_K) RMSNorm + projection GEMVs over raw ggml blocks.
//
// Entries: li_launch_rms_norm_matmul_q, li_launch_fused_rms_norm_qkv_q,
// li_launch_fused_rms_norm_swiglu_q, li_launch_fused_ffn_q,
// li_launch_dequantize; and the in-/out-projection stages of the DeltaNet
// layer decode (li_deltanet.cu) through qgemv_launch().
//
// Design (SIMT path, one x row per pass):
//   * A "unit" is 32 weights of one row: one Q8_0 block, or one 16-byte
//     nibble chunk of a Q4_K super-block (16 low nibbles of sub-block 2i and
//     the 16 high nibbles of sub-block 2i+1). A row has U = K/32 units.
//   * A CTA has RP "row slots" of U (rounded to 32) threads. Thread u of a
//     slot owns unit u of every row the CTA visits, so it keeps the 32 x_norm
//     values of that unit in registers for the whole kernel: x is read once
//     per CTA, never from shared memory in the inner loop.
//   * Weight rows are staged into shared memory by the TMA engine
//     (cp.async.bulk, 1-D) in a ring of S stages of SR rows each, completion
//     tracked by mbarriers (bounded waits). Rows are contiguous in ggml
//     layout, so one stage is one to three bulk copies.
//   * Each thread decodes its unit in registers (byte permutes into float
//     magic numbers; Q4_K scales unpacked per sub-block, the min term folded
//     as dmin*m*sum(x)), reduces with xor-shuffles, and the slot's warps
//     combine through shared memory into an epilogue: plain store, SwiGLU,
//     or the DeltaNet in-projection epilogue (causal conv1d + SiLU with the
//     conv-state shift, so each conv channel has exactly one writer).
//   * The grid is persistent (SM count x resident CTAs); CTAs stride over
//     stages. A launch may be a programmatic dependent launch: weight
//     stages are requested before griddepcontrol.wait, x after it.
#include "li_common.cuh"
#include "li_qgemv.cuh"

LI_DEFINE_TU_STATUS(qgemv)

namespace li {

namespace {

constexpr int kRowsPerThread = 4;     // rows of a stage per row slot
constexpr int kMaxThreads = 1024;
constexpr int kSmemBudget = 100 * 1024;

// ---------------------------------------------------------------------------
// Unit dot products. xr[0..31] are the unit's x values in decode order.
// ---------------------------------------------------------------------------

// Q8_0 block b of a row whose shared-memory copy starts at `srow` (4-byte
// aligned). Reads 9 aligned words; even blocks start on a 4-byte boundary
// (scale in the low half of word 0), odd blocks 2 bytes past one.
__device__ __forceinline__ float dot_q8_0(const uint8_t *srow, int b, const float *xr) {
    const uint32_t off = 34u * (uint32_t)b;
    const uint32_t *w = reinterpret_cast<const uint32_t *>(srow + (off & ~3u));
    uint32_t v[9];
#pragma unroll
    for (int i = 0; i < 9; ++i) v[i] = w[i];
    const uint32_t sh = (off & 2u) ? 32u : 16u;      // odd block: quants start at word 1
    const float d = half_bits_to_float((off & 2u) ? (v[0] >> 16) : v[0]);
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const uint32_t q = __funnelshift_rc(v[j], v[j + 1], sh) ^ 0x80808080u;
#pragma unroll
        for (int bb = 0; bb < 4; ++bb) {
            const float f = __uint_as_float(__byte_perm(q, 0x4B000000u, 0x7540u | bb)) - 8388736.0f;
            acc = fmaf(xr[4 * j + bb], f, acc);
        }
    }
    return d * acc;
}

// Q4_K unit: header word h (d | dmin<<16, then three scale words) and the
// 16-byte nibble chunk q of pair i = c/2. xsum = {sum(xr[0..15]), sum(xr[16..31])}.
__device__ __forceinline__ float dot_q4_k(uint4 h, uint4 q, int c, const float *xr,
                                          float xsum_lo, float xsum_hi) {
    const int i = c >> 1;
    float sc0, m0, sc1, m1;
    q4k_scale_min(h.y, h.z, h.w, 2 * i, sc0, m0);
    q4k_scale_min(h.y, h.z, h.w, 2 * i + 1, sc1, m1);
    const float d = half_bits_to_float(h.x), dmin = half_bits_to_float(h.x >> 16);
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
    float lo = 0.f, hi = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t L = w[j] & 0x0f0f0f0fu;
        const uint32_t H = (w[j] >> 4) & 0x0f0f0f0fu;
#pragma unroll
        for (int bb = 0; bb < 4; ++bb) {
            lo = fmaf(xr[4 * j + bb], byte_to_float(L, bb), lo);
            hi = fmaf(xr[16 + 4 * j + bb], byte_to_float(H, bb), hi);
        }
    }
    return d * (sc0 * lo + sc1 * hi) - dmin * (m0 * xsum_lo + m1 * xsum_hi);
}

// x offsets (elements) of decode position p (0..31) of unit u.
__device__ __forceinline__ int unit_x_index(int wt, int u, int p) {
    if (wt == LI_WTYPE_Q8_0) return 32 * u + p;
    const int sb = u >> 3, c = u & 7, i = c >> 1, h = c & 1;
    return 256 * sb + 64 * i + 16 * h + (p < 16 ? p : 32 + (p - 16));
}

// ---------------------------------------------------------------------------
// The kernel.
// ---------------------------------------------------------------------------
template <int WT, int EPI, int LB>
__global__ void __launch_bounds__(LB)
qgemv_kernel(QGemvArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    const QGemvPlan &p = a.plan;
    const int t = threadIdx.x;
    const int slot = t / p.UP, u = t % p.UP;
    const bool active = u < p.U;
    const int nw = EPI == kEpiSwiGLU ? 2 : 1;
    const size_t rb = p.row_bytes;
    const uint32_t stage_bytes = (uint32_t)(nw * p.SR * rb);

    uint8_t *stages = smem;
    uint64_t *bar = reinterpret_cast<uint64_t *>(smem + (size_t)p.S * stage_bytes);
    float *red = reinterpret_cast<float *>(bar + p.S);          // [SR][warps per slot][2]
    int *abort_flag = reinterpret_cast<int *>(red + p.SR * (p.UP / kWarp) * 2);

    const int wps = p.UP / kWarp;                                // warps per slot
    const int b = blockIdx.y;                                    // x row (batch)
    const int n_stages = (p.total_rows + p.SR - 1) / p.SR;

    // -- issue a stage: rows [r0, r0+SR) of the concatenated row space --
    auto issue = [&](int st, int buf) {
        const int r0 = st * p.SR;
        const int r1 = min(r0 + p.SR, p.total_rows);
        uint8_t *dst = stages + (size_t)buf * stage_bytes;
        mbar_arrive_expect_tx(&bar[buf], (uint32_t)((size_t)nw * (r1 - r0) * rb));
        for (int w = 0; w < nw; ++w) {
            int r = r0;
            while (r < r1) {
                int m = 0, lr = r;
                while (m < a.n_seg - 1 && lr >= a.seg_rows[m]) lr -= a.seg_rows[m++];
                const int take = min(r1 - r, a.seg_rows[m] - lr);
                const uint8_t *src = reinterpret_cast<const uint8_t *>(a.W[w == 0 ? m : 1]) +
                                     (size_t)lr * rb;
                bulk_g2s(dst + ((size_t)w * p.SR + (r - r0)) * rb, src, (uint32_t)(take * rb),
                         &bar[buf]);
                r += take;
            }
        }
    };

    if (t == 0) {
        for (int s = 0; s < p.S; ++s) mbar_init(&bar[s], 1);
        fence_mbar_init();
        *abort_flag = 0;
    }
    __syncthreads();
    if (t == 0) {
        for (int s = 0; s < p.S; ++s) {
            const int st = blockIdx.x + s * gridDim.x;
            if (st < n_stages) issue(st, s);
        }
    }
    // Let a dependent launch start its own weight-independent prologue.
    grid_dep_launch_dependents();

    // x depends on the previous kernel in the stream; weights do not.
    grid_dep_wait();

    // -- x_norm of this thread's unit into registers --
    float xr[32];
    float xs_lo = 0.f, xs_hi = 0.f;
    {
        const float *xrow = a.x + (size_t)b * a.x_stride;
        float sq = 0.f;
#pragma unroll
        for (int q = 0; q < 32; ++q) {
            const float v = active ? xrow[unit_x_index(WT, u, q)] : 0.f;
            xr[q] = v;
            sq = fmaf(v, v, sq);
        }
        if (a.gamma) {
            sq = warp_sum(slot == 0 ? sq : 0.f);
            __shared__ float sred[kMaxThreads / kWarp];
            if ((t % kWarp) == 0) sred[t / kWarp] = sq;
            __syncthreads();
            float tot = 0.f;
            for (int w = 0; w < wps; ++w) tot += sred[w];
            const float r = rsqrtf(tot / (float)a.K + a.eps);
#pragma unroll
            for (int q = 0; q < 32; ++q)
                xr[q] = active ? xr[q] * a.gamma[unit_x_index(WT, u, q)] * r : 0.f;
        }
#pragma unroll
        for (int q = 0; q < 16; ++q) {
            xs_lo += xr[q];
            xs_hi += xr[16 + q];
        }
    }

    int it = 0;
    for (;; ++it) {
        const int st = blockIdx.x + it * gridDim.x;
        if (st >= n_stages) break;
        const int buf = it % p.S;
        if (!mbar_wait(&bar[buf], (uint32_t)((it / p.S) & 1))) atomicExch(abort_flag, 1);
        const uint8_t *sbuf = stages + (size_t)buf * stage_bytes;
        const int r0 = st * p.SR;

        // partial dot products of this thread's unit over its rows
        float part[kRowsPerThread][2];
#pragma unroll
        for (int j = 0; j < kRowsPerThread; ++j) {
            const int lr = slot + p.RP * j;
#pragma unroll
            for (int w = 0; w < 2; ++w) {
                part[j][w] = 0.f;
                if (w < nw && active && lr < p.SR && r0 + lr < p.total_rows && !*abort_flag) {
                    const uint8_t *srow = sbuf + ((size_t)w * p.SR + lr) * rb;
                    if (WT == LI_WTYPE_Q8_0) {
                        part[j][w] = dot_q8_0(srow, u, xr);
                    } else {
                        const int sb = u >> 3, c = u & 7;
                        const uint4 h = *reinterpret_cast<const uint4 *>(srow + 144 * sb);
                        const uint4 q = *reinterpret_cast<const uint4 *>(srow + 144 * sb + 16 + 16 * c);
                        part[j][w] = dot_q4_k(h, q, c, xr, xs_lo, xs_hi);
                    }
                }
            }
        }
#pragma unroll
        for (int j = 0; j < kRowsPerThread; ++j)
#pragma unroll
            for (int w = 0; w < 2; ++w) part[j][w] = warp_sum(part[j][w]);
        if ((t % kWarp) == 0) {
            const int wi = u / kWarp;
#pragma unroll
            for (int j = 0; j < kRowsPerThread; ++j) {
                const int lr = slot + p.RP * j;
                if (lr < p.SR) {
                    red[(lr * wps + wi) * 2 + 0] = part[j][0];
                    red[(lr * wps + wi) * 2 + 1] = part[j][1];
                }
            }
        }
        __syncthreads();                 // stage buffer free, partials visible
        if (*abort_flag) break;
        if (t == 0) {
            const int nst = blockIdx.x + (it + p.S) * gridDim.x;
            if (nst < n_stages) issue(nst, buf);
        }
        if (t < p.SR && r0 + t < p.total_rows) {
            float s0 = 0.f, s1 = 0.f;
            for (int w = 0; w < wps; ++w) {
                s0 += red[(t * wps + w) * 2 + 0];
                s1 += red[(t * wps + w) * 2 + 1];
            }
            const int row = r0 + t;
            if (EPI == kEpiSwiGLU) {
                a.dst[0][(size_t)b * a.dst_stride[0] + row] = silu(s0) * s1;
            } else if (EPI == kEpiStore) {
                int m = 0, lr = row;
                while (m < a.n_seg - 1 && lr >= a.seg_rows[m]) lr -= a.seg_rows[m++];
                a.dst[m][(size_t)b * a.dst_stride[m] + lr] = s0;
            } else {  // kEpiConv: DeltaNet in-projection epilogue
                float out = s0;
                if (row < a.conv_channels) {
                    float *cs = a.conv_state + ((size_t)b * a.conv_channels + row) * 3;
                    const float4 cw = *reinterpret_cast<const float4 *>(a.conv_w + 4 * (size_t)row);
                    const float c0 = cs[0], c1 = cs[1], c2 = cs[2];
                    const float acc = fmaf(cw.x, c0, fmaf(cw.y, c1, fmaf(cw.z, c2, cw.w * s0)));
                    cs[0] = c1;
                    cs[1] = c2;
                    cs[2] = s0;
                    out = silu(acc);
                }
                a.dst[0][(size_t)b * a.dst_stride[0] + row] = out;
            }
        }
        __syncthreads();                 // red reused next iteration
    }
    if (*abort_flag && t == 0) {
        // A wait gave up at iteration `it`: stages it .. it+S-1 were issued
        // and not consumed. Drain them (bounded) before the CTA's shared
        // memory is released.
        for (int j = it; j < it + p.S; ++j)
            if (blockIdx.x + j * gridDim.x < n_stages) mbar_wait(&bar[j % p.S], (uint32_t)((j / p.S) & 1));
    }
}

}  // namespace

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
int qgemv_plan(int wtype, int K, int total_rows, int epi, QGemvPlan *p) {
    if (wtype != LI_WTYPE_Q8_0 && wtype != LI_WTYPE_Q4_K) return LI_ERR_UNSUPPORTED;
    const size_t rb = li_row_bytes(wtype, K);
    if (!rb || K % 256) return LI_ERR_BAD_SHAPE;               // bulk copies need 16-byte rows
    p->U = K / 32;
    p->UP = (p->U + kWarp - 1) / kWarp * kWarp;
    if (p->UP > kMaxThreads) return LI_ERR_BAD_SHAPE;
    p->RP = p->UP >= 256 ? 1 : 256 / p->UP;
    p->SR = p->RP * kRowsPerThread;
    p->row_bytes = rb;
    p->total_rows = total_rows;
    const int nw = epi == kEpiSwiGLU ? 2 : 1;
    size_t stage = (size_t)nw * p->SR * rb;
    p->S = (int)(kSmemBudget / stage);
    if (p->S > 4) p->S = 4;
    if (p->S < 2) p->S = 2;
    if (p->S * stage > 200 * 1024) return LI_ERR_BAD_SHAPE;
    p->threads = p->UP * p->RP;
    p->smem = p->S * stage + p->S * sizeof(uint64_t) + (size_t)p->SR * (p->UP / kWarp) * 2 * 4 + 16;
    return 0;
}

template <int WT, int EPI>
static int launch_t(const QGemvArgs &a, int n_rows, cudaStream_t stream, bool pdl) {
    auto kern = a.plan.threads <= 512 ? qgemv_kernel<WT, EPI, 512> : qgemv_kernel<WT, EPI, 1024>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)a.plan.smem);
    if (e != cudaSuccess) return (int)e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, a.plan.threads, a.plan.smem);
    if (e != cudaSuccess) return (int)e;
    if (per_sm < 1) return LI_ERR_BAD_SHAPE;
    const int n_stages = (a.plan.total_rows + a.plan.SR - 1) / a.plan.SR;
    int grid = num_sms() * per_sm;
    if (grid > n_stages) grid = n_stages;
    e = launch_pdl(kern, dim3(grid, n_rows), dim3(a.plan.threads), a.plan.smem, stream, pdl, a);
    return (int)e;
}

int qgemv_launch(const QGemvArgs &a, int n_rows, cudaStream_t stream, bool pdl) {
    const int wt = a.wtype;
    switch (a.epi) {
    case kEpiStore:
        return wt == LI_WTYPE_Q8_0 ? launch_t<LI_WTYPE_Q8_0, kEpiStore>(a, n_rows, stream, pdl)
                                   : launch_t<LI_WTYPE_Q4_K, kEpiStore>(a, n_rows, stream, pdl);
    case kEpiSwiGLU:
        return wt == LI_WTYPE_Q8_0 ? launch_t<LI_WTYPE_Q8_0, kEpiSwiGLU>(a, n_rows, stream, pdl)
                                   : launch_t<LI_WTYPE_Q4_K, kEpiSwiGLU>(a, n_rows, stream, pdl);
    case kEpiConv:
        return wt == LI_WTYPE_Q8_0 ? launch_t<LI_WTYPE_Q8_0, kEpiConv>(a, n_rows, stream, pdl)
                                   : launch_t<LI_WTYPE_Q4_K, kEpiConv>(a, n_rows, stream, pdl);
    default:
        return LI_ERR_BAD_ARG;
    }
}

// ---------------------------------------------------------------------------
// Block decode (ggml to_float), bit-exact with gguf-py: products and the
// subtraction are rounded separately (__fmul_rn / __fsub_rn forbid FMA).
// ---------------------------------------------------------------------------
namespace {

__global__ void dequant_q8_0_kernel(const uint8_t *__restrict__ src, float *__restrict__ dst,
                                    int64_t nblocks) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;   // one value each
    const int64_t blk = i >> 5;
    if (blk >= nblocks) return;
    const uint8_t *bp = src + blk * 34;
    const uint32_t dh = (uint32_t)bp[0] | ((uint32_t)bp[1] << 8);
    const float d = half_bits_to_float(dh);
    const int8_t q = (int8_t)bp[2 + (i & 31)];
    dst[i] = __fmul_rn((float)q, d);
}

__global__ void dequant_q4_k_kernel(const uint8_t *__restrict__ src, float *__restrict__ dst,
                                    int64_t nblocks) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t blk = i >> 8;
    if (blk >= nblocks) return;
    const uint8_t *bp = src + blk * 144;
    const int pos = (int)(i & 255), j = pos >> 5, l = pos & 31;
    const uint32_t d16 = (uint32_t)bp[0] | ((uint32_t)bp[1] << 8);
    const uint32_t m16 = (uint32_t)bp[2] | ((uint32_t)bp[3] << 8);
    const uint32_t *s = reinterpret_cast<const uint32_t *>(bp + 4);  // bp + 4 is 4-byte aligned
    float sc, mn;
    q4k_scale_min(s[0], s[1], s[2], j, sc, mn);
    const float dl = __fmul_rn(half_bits_to_float(d16), sc);
    const float ml = __fmul_rn(half_bits_to_float(m16), mn);
    const uint8_t byte = bp[16 + 32 * (j >> 1) + l];
    const float q = (float)((j & 1) ? (byte >> 4) : (byte & 15));
    dst[i] = __fsub_rn(__fmul_rn(dl, q), ml);
}

}  // namespace
}  // namespace li

using namespace li;

static int common_q_checks(int wtype, const void *x, const void *W, const void *dst, int K, int N,
                           int n_rows) {
    if (!x || !W || !dst || K <= 0 || N < 0 || n_rows < 0) return LI_ERR_BAD_ARG;
    if (wtype != LI_WTYPE_Q8_0 && wtype != LI_WTYPE_Q4_K) return LI_ERR_UNSUPPORTED;
    if (!aligned16(W)) return LI_ERR_MISALIGNED;
    return 0;
}

extern "C" {

int li_launch_dequantize(int wtype, const void *src, float *dst, int64_t n, void *stream) {
    if (!src || !dst || n < 0) return LI_ERR_BAD_ARG;
    if (n == 0) return 0;
    const cudaStream_t s = (cudaStream_t)stream;
    const int64_t blocks = (n + 255) / 256;
    if (wtype == LI_WTYPE_Q8_0) {
        if (n % 32) return LI_ERR_BAD_SHAPE;
        dequant_q8_0_kernel<<<(unsigned)blocks, 256, 0, s>>>((const uint8_t *)src, dst, n / 32);
    } else if (wtype == LI_WTYPE_Q4_K) {
        if (n % 256) return LI_ERR_BAD_SHAPE;
        if (((uintptr_t)src & 3u) != 0) return LI_ERR_MISALIGNED;
        dequant_q4_k_kernel<<<(unsigned)blocks, 256, 0, s>>>((const uint8_t *)src, dst, n / 256);
    } else {
        return LI_ERR_UNSUPPORTED;
    }
    return launch_status();
}

int li_launch_rms_norm_matmul_q(int wtype, const float *x, const float *gamma, const void *W,
                                float *dst, int K, int N, int n_rows, float eps, void *stream) {
    int rc = common_q_checks(wtype, x, W, dst, K, N, n_rows);
    if (rc) return rc;
    if (N == 0 || n_rows == 0) return 0;
    QGemvArgs a = {};
    a.wtype = wtype; a.epi = kEpiStore;
    if ((rc = qgemv_plan(wtype, K, N, kEpiStore, &a.plan))) return rc;
    a.x = x; a.x_stride = K; a.gamma = gamma; a.K = K; a.eps = eps;
    a.n_seg = 1; a.W[0] = W; a.seg_rows[0] = N; a.dst[0] = dst; a.dst_stride[0] = N;
    return qgemv_launch(a, n_rows, (cudaStream_t)stream, false);
}

int li_launch_fused_rms_norm_qkv_q(int wtype, const float *x, const float *gamma, const void *Wq,
                                   const void *Wk, const void *Wv, float *q, float *k, float *v,
                                   int K, int Nq, int Nk, int Nv, int n_rows, float eps,
                                   void *stream) {
    int rc = common_q_checks(wtype, x, Wq, q, K, Nq, n_rows);
    if (!rc) rc = common_q_checks(wtype, x, Wk, k, K, Nk, n_rows);
    if (!rc) rc = common_q_checks(wtype, x, Wv, v, K, Nv, n_rows);
    if (rc) return rc;
    if (!gamma) return LI_ERR_BAD_ARG;
    const int total = Nq + Nk + Nv;
    if (total == 0 || n_rows == 0) return 0;
    QGemvArgs a = {};
    a.wtype = wtype; a.epi = kEpiStore;
    if ((rc = qgemv_plan(wtype, K, total, kEpiStore, &a.plan))) return rc;
    a.x = x; a.x_stride = K; a.gamma = gamma; a.K = K; a.eps = eps;
    a.n_seg = 3;
    a.W[0] = Wq; a.W[1] = Wk; a.W[2] = Wv;
    a.seg_rows[0] = Nq; a.seg_rows[1] = Nk; a.seg_rows[2] = Nv;
    a.dst[0] = q; a.dst[1] = k; a.dst[2] = v;
    a.dst_stride[0] = Nq; a.dst_stride[1] = Nk; a.dst_stride[2] = Nv;
    return qgemv_launch(a, n_rows, (cudaStream_t)stream, false);
}

int li_launch_fused_rms_norm_swiglu_q(int wtype, const float *x, const float *gamma,
                                      const void *Wg, const void *Wu, float *h, int K, int N,
                                      int n_rows, float eps, void *stream) {
    int rc = common_q_checks(wtype, x, Wg, h, K, N, n_rows);
    if (!rc) rc = common_q_checks(wtype, x, Wu, h, K, N, n_rows);
    if (rc) return rc;
    if (N == 0 || n_rows == 0) return 0;
    QGemvArgs a = {};
    a.wtype = wtype; a.epi = kEpiSwiGLU;
    if ((rc = qgemv_plan(wtype, K, N, kEpiSwiGLU, &a.plan))) return rc;
    a.x = x; a.x_stride = K; a.gamma = gamma; a.K = K; a.eps = eps;
    a.n_seg = 1; a.W[0] = Wg; a.W[1] = Wu; a.seg_rows[0] = N;
    a.dst[0] = h; a.dst_stride[0] = N;
    return qgemv_launch(a, n_rows, (cudaStream_t)stream, false);
}

size_t li_fused_ffn_workspace_size(int N, int n_rows) {
    if (N <= 0 || n_rows <= 0) return 0;
    return ((size_t)N * n_rows * sizeof(float) + 255) / 256 * 256;
}

int li_launch_fused_ffn_q(int wtype, const float *x, const float *gamma, const void *Wg,
                          const void *Wu, const void *Wd, float *y, int K, int N, int n_rows,
                          float eps, void *workspace, size_t workspace_bytes, void *stream) {
    int rc = common_q_checks(wtype, x, Wg, y, K, N, n_rows);
    if (!rc) rc = common_q_checks(wtype, x, Wu, y, K, N, n_rows);
    if (!rc) rc = common_q_checks(wtype, x, Wd, y, N, K, n_rows);
    if (rc) return rc;
    if (N == 0 || n_rows == 0) return 0;
    if (!workspace || workspace_bytes < li_fused_ffn_workspace_size(N, n_rows))
        return LI_ERR_WORKSPACE;
    float *h = (float *)workspace;
    QGemvArgs a = {};
    a.wtype = wtype; a.epi = kEpiSwiGLU;
    if ((rc = qgemv_plan(wtype, K, N, kEpiSwiGLU, &a.plan))) return rc;
    a.x = x; a.x_stride = K; a.gamma = gamma; a.K = K; a.eps = eps;
    a.n_seg = 1; a.W[0] = Wg; a.W[1] = Wu; a.seg_rows[0] = N;
    a.dst[0] = h; a.dst_stride[0] = N;
    if ((rc = qgemv_launch(a, n_rows, (cudaStream_t)stream, false))) return rc;
    QGemvArgs d = {};
    d.wtype = wtype; d.epi = kEpiStore;
    if ((rc = qgemv_plan(wtype, N, K, kEpiStore, &d.plan))) return rc;
    d.x = h; d.x_stride = N; d.gamma = nullptr; d.K = N; d.eps = 0.f;
    d.n_seg = 1; d.W[0] = Wd; d.seg_rows[0] = K; d.dst[0] = y; d.dst_stride[0] = K;
    return qgemv_launch(d, n_rows, (cudaStream_t)stream, true);
}

}  // extern "C"
