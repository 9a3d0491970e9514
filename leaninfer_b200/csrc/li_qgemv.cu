// Quantized (Q8_0 / Q4_K) RMSNorm + projection GEMVs over raw ggml blocks.
//
// Entries: li_launch_rms_norm_matmul_q, li_launch_fused_rms_norm_qkv_q,
// li_launch_fused_rms_norm_swiglu_q, li_launch_fused_ffn_q,
// li_launch_dequantize; and the in-/out-projection stages of the DeltaNet
// layer decode (li_deltanet.cu) through qgemv_launch().
//
// Design (SIMT path, one x row per CTA row):
//   * A "unit" is a fixed slice of a row: one Q8_0 block (32 weights) or one
//     Q4_K sub-block pair (64 weights: the 32 nibble bytes of pair i hold
//     sub-block 2i in their low and 2i+1 in their high nibbles). A row has U
//     units. A CTA has RP "row slots" of U (rounded up to 32) threads; thread
//     u of a slot owns unit u of every row the CTA visits and keeps that
//     unit's x_norm values in registers for the whole kernel.
//   * Weight rows are staged into shared memory by the TMA engine
//     (cp.async.bulk, 1-D) in a ring of S stages of SR rows each, completion
//     tracked by mbarriers with bounded waits. Rows are contiguous in ggml
//     layout, so a stage is one to three bulk copies.
//   * Integer dot products: each thread quantizes its (fixed) x slice once,
//     per 32-value sub-block, to int16 with scale max|x|/32767 (error at
//     most 1.5e-5 of the sub-block's max |x|), and multiplies it against the
//     codes with dp2a (two int16 x int8 products per instruction, exact
//     int32 sums). Q8_0 code words feed dp2a as they are; Q4_K needs one mask
//     and one shift per 8 nibbles. The unit's partial is rescaled in fp32 by
//     the block scale(s) and the x scale; the Q4_K min term uses the fp32
//     sum of x.
//   * Each thread reduces its R rows with a butterfly transpose over the
//     warp (R-1 + log2(32/R) shuffles for R rows), warps of a slot combine
//     through double-buffered shared memory, one barrier per stage, into an
//     epilogue: plain store, SwiGLU, or the DeltaNet in-projection epilogue
//     (causal conv1d + SiLU with the conv-state shift, one writer per
//     channel).
//   * The grid is persistent (SM count x resident CTAs); CTAs stride over
//     stages. A launch may be a programmatic dependent launch: weight stages
//     are requested before griddepcontrol.wait, x after it.
//   * Up to 8 x rows with K a multiple of 32 units (at most 2 units per
//     lane; 4 Q8_0 units for one x row) take qgemv_row_kernel instead: no
//     staging, a warp per group of adjacent rows, weights loaded straight
//     into registers and multiplied with every x row.
#include "li_common.cuh"
#include "li_qgemv.cuh"
#include "li_tcgemm.cuh"

#include <mutex>
#include <vector>

LI_DEFINE_TU_STATUS(qgemv)

namespace li {

namespace {

constexpr int kMaxThreads = 512;      // 64-weight units: K <= 16384 (Q8_0), 32768 (Q4_K)
constexpr int kStageTarget = 40 * 1024;   // bytes of weight rows per stage
constexpr int kSmemBudget = 112 * 1024;   // stages per CTA (two CTAs per SM)

// Weights per unit.
__host__ __device__ constexpr int unit_weights(int wt) { return wt == LI_WTYPE_Q8_0 ? 32 : 64; }

// Q8_0 block dot product from the block's 9 aligned words (starting at the
// 4-byte boundary at or below the block): even blocks start on the boundary
// (scale in the low half of word 0), odd blocks 2 bytes past it. xq[k] =
// int16 pair (x[2k], x[2k+1]) of the block, xscale its quantization step.
__device__ __forceinline__ float dot_q8_0_words(const uint32_t (&v)[9], bool odd, const int *xq, float xscale) {
    const uint32_t sh = odd ? 32u : 16u;
    const float d = half_bits_to_float(odd ? (v[0] >> 16) : v[0]);
    int acc = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int q = (int)__funnelshift_rc(v[j], v[j + 1], sh);
        acc = __dp2a_lo(xq[2 * j], q, acc);
        acc = __dp2a_hi(xq[2 * j + 1], q, acc);
    }
    return d * xscale * (float)acc;
}

// Q8_0 block u of a row whose shared-memory copy starts at `srow` (4-byte aligned).
__device__ __forceinline__ float dot_q8_0(const uint8_t *srow, int u, const int *xq, float xscale) {
    const uint32_t off = 34u * (uint32_t)u;
    const uint32_t *w = reinterpret_cast<const uint32_t *>(srow + (off & ~3u));
    uint32_t v[9];
#pragma unroll
    for (int i = 0; i < 9; ++i) v[i] = w[i];
    return dot_q8_0_words(v, (off & 2u) != 0, xq, xscale);
}

// Integer dot of the 32 nibbles of one sub-block of a pair (low nibbles of
// the pair's 8 words for sub-block 2i, shift 0; high nibbles for 2i+1,
// shift 4) with its int16 x pairs.
__device__ __forceinline__ int q4k_nibble_dot(const uint32_t (&w)[8], uint32_t shift, const int *xq) {
    int acc = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int q = (int)((w[j] >> shift) & 0x0f0f0f0fu);   // positions 4j..4j+3
        acc = __dp2a_lo(xq[2 * j], q, acc);
        acc = __dp2a_hi(xq[2 * j + 1], q, acc);
    }
    return acc;
}

// Value of pair i from its two integer dots acc0 / acc1 and the header h.
__device__ __forceinline__ float q4k_combine(uint4 h, int i, int acc0, int acc1, float xs0, float xs1,
                                             float sum0, float sum1) {
    const uint32_t bsh = 16u * (uint32_t)(i & 1);
    const uint32_t a0 = h.y >> bsh, a1 = h.z >> bsh, a2 = h.w >> bsh;
    uint32_t sc0, sc1, m0, m1;
    if (i < 2) {
        sc0 = a0 & 63u; sc1 = (a0 >> 8) & 63u; m0 = a1 & 63u; m1 = (a1 >> 8) & 63u;
    } else {
        sc0 = (a2 & 15u) | ((a0 >> 2) & 48u);
        sc1 = ((a2 >> 8) & 15u) | ((a0 >> 10) & 48u);
        m0 = ((a2 >> 4) & 15u) | ((a1 >> 2) & 48u);
        m1 = ((a2 >> 12) & 15u) | ((a1 >> 10) & 48u);
    }
    const float d = half_bits_to_float(h.x), dmin = half_bits_to_float(h.x >> 16);
    return d * fmaf((float)sc0 * xs0, (float)acc0, (float)sc1 * xs1 * (float)acc1) -
           dmin * fmaf((float)m0, sum0, (float)m1 * sum1);
}

// Q4_K sub-block pair i of a super-block: header h = {d | dmin<<16, scale
// bytes 0-3, 4-7, 8-11}, nibble bytes q0 (0-15) and q1 (16-31) of the pair.
// xq0/xq1 = int16 pairs of sub-blocks 2i / 2i+1, xs0/xs1 their steps,
// sum0/sum1 their fp32 sums of x.
__device__ __forceinline__ float dot_q4_k(uint4 h, uint4 q0, uint4 q1, int i, const int *xq0,
                                          const int *xq1, float xs0, float xs1, float sum0,
                                          float sum1) {
    const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
    return q4k_combine(h, i, q4k_nibble_dot(w, 0, xq0), q4k_nibble_dot(w, 4, xq1), xs0, xs1, sum0, sum1);
}

// Quantize 32 fp32 values to int16 pairs with step max|v|/32767; returns
// the step (0 for an all-zero slice).
__device__ __forceinline__ float quantize32_s16(const float *v, int *xq) {
    float mx = 0.f;
#pragma unroll
    for (int k = 0; k < 32; ++k) mx = fmaxf(mx, fabsf(v[k]));
    const float step = mx / 32767.0f;
    const float inv = mx > 0.f ? 32767.0f / mx : 0.f;
#pragma unroll
    for (int k = 0; k < 16; ++k) {
        const int a = __float2int_rn(v[2 * k] * inv);
        const int b = __float2int_rn(v[2 * k + 1] * inv);
        xq[k] = (a & 0xffff) | (b << 16);
    }
    return step;
}

// Butterfly transpose-reduction of V values per lane over the warp: after
// it, lane l holds the warp sum of value index (l >> (5 - log2 V)) & (V-1).
template <int V>
__device__ __forceinline__ float warp_transpose_reduce(float (&v)[V], int lane) {
    int cur = V;
#pragma unroll
    for (int o = 16; cur > 1; o >>= 1) {
        const bool upper = (lane & o) != 0;
        const int half = cur >> 1;
#pragma unroll
        for (int i = 0; i < half; ++i) {
            const float send = upper ? v[i] : v[i + half];
            const float keep = upper ? v[i + half] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
        cur = half;
    }
    float r = v[0];
    constexpr int lv = V == 1 ? 0 : V == 2 ? 1 : V == 4 ? 2 : V == 8 ? 3 : 4;
#pragma unroll
    for (int o = 16 >> lv; o > 0; o >>= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
    return r;
}

// ---------------------------------------------------------------------------
// The kernel. R = rows per slot per stage, NW = weight streams (2: SwiGLU).
// ---------------------------------------------------------------------------
template <int WT, int EPI, int LB, int R>
__global__ void __launch_bounds__(LB)
qgemv_kernel(QGemvArgs a) {
    constexpr int NW = EPI == kEpiSwiGLU ? 2 : 1;
    constexpr int V = NW * R;                         // values per thread per stage
    constexpr int UW = unit_weights(WT);              // weights per unit
    extern __shared__ __align__(16) uint8_t smem[];
    const QGemvPlan &p = a.plan;
    const int t = threadIdx.x, lane = t % kWarp;
    const int slot = t / p.UP, u = t % p.UP;
    const bool active = u < p.U;
    const size_t rb = p.row_bytes;
    const uint32_t stage_bytes = (uint32_t)(NW * p.SR * rb);
    const int wps = p.UP / kWarp;                     // warps per slot
    const int XB = p.XB;                              // buffers that first stage x

    uint8_t *stages = smem;
    uint64_t *bar = reinterpret_cast<uint64_t *>(smem + (size_t)p.S * stage_bytes);
    float *red = reinterpret_cast<float *>(bar + p.S);   // [2][SR][wps][NW]
    int *abort_flag = reinterpret_cast<int *>(red + 2 * p.SR * wps * NW);
    __shared__ float sred[kMaxThreads / kWarp];

    const int b = blockIdx.y;                         // x row (batch)
    const int n_stages = (p.total_rows + p.SR - 1) / p.SR;

    // Pipeline slots: virtual iteration v uses buffer v % S and, for v >= XB,
    // holds weight stage stage_of(v). Virtual iterations 0..XB-1 are not
    // weight stages: their buffers stage x while weight stages XB..S-1 are
    // already in flight. Buffer v % S has completed (v / S) - (v % S < XB)
    // bulk-copy phases before the copy of iteration v.
    auto stage_of = [&](int v) { return (int)blockIdx.x + (v - XB) * (int)gridDim.x; };
    auto parity_of = [&](int v) { return (uint32_t)(((v / p.S) - ((v % p.S) < XB ? 1 : 0)) & 1); };

    auto issue = [&](int v) {
        const int st = stage_of(v);
        const int buf = v % p.S;
        const int r0 = st * p.SR;
        const int r1 = min(r0 + p.SR, p.total_rows);
        uint8_t *dst = stages + (size_t)buf * stage_bytes;
        mbar_arrive_expect_tx(&bar[buf], (uint32_t)((size_t)NW * (r1 - r0) * rb));
        for (int w = 0; w < NW; ++w) {
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
        for (int v = XB; v < p.S; ++v)
            if (stage_of(v) < n_stages) issue(v);
    }
    // x depends on the previous kernel in the stream; weights do not. A
    // dependent launch may start its own prologue once this kernel's
    // predecessor has completed (the recurrence after a layer's first GEMV
    // reads its state before its own wait).
    grid_dep_wait();
    grid_dep_launch_dependents();

    // -- x (times gamma) into buffers 0..XB-1, coalesced, padded by one
    //    float per unit so the per-unit reads below are conflict free --
    float *xs = reinterpret_cast<float *>(stages);
    float rnorm = 1.0f;
    {
        const float4 *x4 = reinterpret_cast<const float4 *>(a.x + (size_t)b * a.x_stride);
        const float4 *g4 = reinterpret_cast<const float4 *>(a.gamma);
        float sq = 0.f;
        for (int i = t; i < a.K / 4; i += blockDim.x) {
            float4 v = x4[i];
            sq = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, sq))));
            if (a.gamma) {
                const float4 g = g4[i];
                v.x *= g.x; v.y *= g.y; v.z *= g.z; v.w *= g.w;
            }
            const int k = 4 * i, kp = k + k / UW;
            xs[kp] = v.x; xs[kp + 1] = v.y; xs[kp + 2] = v.z; xs[kp + 3] = v.w;
        }
        sq = warp_sum(sq);
        if (lane == 0) sred[t / kWarp] = sq;
        __syncthreads();
        if (a.gamma) {
            float tot = 0.f;
            for (int w = 0; w < (int)(blockDim.x / kWarp); ++w) tot += sred[w];
            rnorm = rsqrtf(tot / (float)a.K + a.eps);
        }
    }

    // -- this thread's unit: x_norm quantized to int16 per 32-value sub-block --
    constexpr int NSUB = UW / 32;                     // sub-blocks per unit
    int xq[NSUB][16];
    float xstep[NSUB], xsum[NSUB];
    {
        const float *xu = xs + (size_t)(active ? u : 0) * (UW + 1);
#pragma unroll
        for (int sb = 0; sb < NSUB; ++sb) {
            float v[32];
            float sm = 0.f;
#pragma unroll
            for (int k = 0; k < 32; ++k) {
                v[k] = active ? xu[32 * sb + k] * rnorm : 0.f;
                sm += v[k];
            }
            xsum[sb] = sm;
            xstep[sb] = quantize32_s16(v, xq[sb]);
        }
    }
    __syncthreads();                     // x buffers free
    if (t == 0) {
        for (int v = p.S; v < p.S + XB; ++v)
            if (stage_of(v) < n_stages) issue(v);
    }

    int v = XB;
    for (;; ++v) {
        const int st = stage_of(v);
        if (st >= n_stages) break;
        const int buf = v % p.S;
        if (!mbar_wait(&bar[buf], parity_of(v))) atomicExch(abort_flag, 1);
        const uint8_t *sbuf = stages + (size_t)buf * stage_bytes;
        const int r0 = st * p.SR;

        float part[V];
#pragma unroll
        for (int j = 0; j < R; ++j) {
            const int lr = slot + p.RP * j;
            const bool ok = active && r0 + lr < p.total_rows;
#pragma unroll
            for (int w = 0; w < NW; ++w) {
                float val = 0.f;
                if (ok) {
                    const uint8_t *srow = sbuf + ((size_t)w * p.SR + lr) * rb;
                    if (WT == LI_WTYPE_Q8_0) {
                        val = dot_q8_0(srow, u, xq[0], xstep[0]);
                    } else {
                        const uint8_t *blk = srow + 144 * (u >> 2);
                        const uint4 h = *reinterpret_cast<const uint4 *>(blk);
                        const uint4 q0 = *reinterpret_cast<const uint4 *>(blk + 16 + 32 * (u & 3));
                        const uint4 q1 = *reinterpret_cast<const uint4 *>(blk + 32 + 32 * (u & 3));
                        val = dot_q4_k(h, q0, q1, u & 3, xq[0], xq[NSUB - 1], xstep[0], xstep[NSUB - 1],
                                       xsum[0], xsum[NSUB - 1]);
                    }
                }
                part[w * R + j] = val;
            }
        }
        const float sum = warp_transpose_reduce<V>(part, lane);
        float *rb2 = red + (size_t)(v & 1) * p.SR * wps * NW;
        constexpr int lv = V == 1 ? 0 : V == 2 ? 1 : V == 4 ? 2 : V == 8 ? 3 : 4;
        if ((lane & ((32 >> lv) - 1)) == 0) {
            const int vi = (lane >> (5 - lv)) & (V - 1);
            const int w = vi / R, j = vi % R;
            const int lr = slot + p.RP * j;
            rb2[(lr * wps + u / kWarp) * NW + w] = sum;
        }
        __syncthreads();                 // stage buffer free, partials visible
        if (*abort_flag) break;
        if (t == 0 && stage_of(v + p.S) < n_stages) issue(v + p.S);
        if (t < p.SR && r0 + t < p.total_rows) {
            float s0 = 0.f, s1 = 0.f;
            for (int w = 0; w < wps; ++w) {
                s0 += rb2[(t * wps + w) * NW];
                if (NW == 2) s1 += rb2[(t * wps + w) * NW + 1];
            }
            const int row = r0 + t;
            if (EPI == kEpiSwiGLU) {
                a.dst[0][(size_t)b * a.dst_stride[0] + row] = silu(s0) * s1;
            } else if (EPI == kEpiStore) {
                int m = 0, lr = row;
                while (m < a.n_seg - 1 && lr >= a.seg_rows[m]) lr -= a.seg_rows[m++];
                float *d = m == 0 ? a.dst[0] : (m == 1 ? a.dst[1] : a.dst[2]);
                const int ds = m == 0 ? a.dst_stride[0] : (m == 1 ? a.dst_stride[1] : a.dst_stride[2]);
                float *o = d + (size_t)b * ds + lr;
                *o = a.accumulate ? *o + s0 : s0;
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
    }
    if (*abort_flag && t == 0) {
        // A wait gave up at virtual iteration v: iterations v .. v+S-1 were
        // issued and not consumed. Drain them (bounded) before the CTA's
        // shared memory is released.
        for (int j = v; j < v + p.S; ++j)
            if (stage_of(j) < n_stages) mbar_wait(&bar[j % p.S], parity_of(j));
    }
}


// ---------------------------------------------------------------------------
// A few batch rows (nb <= NB <= 8): a warp owns whole weight rows and lane l
// handles units l, l+32, ... (UPL of them) of each. The CTA quantizes the nb
// x rows once into shared memory (int16 pairs in [row][sub-block][16-byte
// chunk][unit] order, so a warp's 16-byte reads of one chunk are
// conflict-free), and lanes read their weight units straight from global
// memory (the warp's loads of a row cover one contiguous range). A warp
// holds the weights of R adjacent rows (one contiguous range of the matrix)
// in registers and multiplies them with every x row: the first R rows are
// loaded before the wait on the previous kernel (weights are constant), the
// next R rows as soon as the current ones are multiplied, so the loads
// overlap the reductions and epilogues. Lane rr * NB + b finishes (row rr,
// x row b); in the in-projection epilogue it fetches its conv state and
// taps one iteration ahead. Same quantization and unit dot products as
// qgemv_kernel.
// ---------------------------------------------------------------------------
constexpr int kRowThreads = 512;
constexpr int kRowMaxBatch = 8;

// Read-only weight loads.
__device__ __forceinline__ uint4 ldg_nc16(const uint8_t *p) {
    uint4 v;
    asm("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
        : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}
__device__ __forceinline__ uint32_t ldg_nc4(const uint8_t *p) {
    uint32_t v;
    asm("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}

// 32-bit words a lane holds per unit of one weight row.
__host__ __device__ constexpr int row_unit_words(int wt) { return wt == LI_WTYPE_Q8_0 ? 9 : 12; }

// Rows a warp keeps in flight: about 72 registers of weights for one x
// row; for several, about 60 registers of weights and accumulators (40 with
// one unit per lane, where more rows share each x read). At least 1, at
// most 4, and R * NB <= 32 lanes.
__host__ __device__ constexpr int row_batch_raw(int wt, int nw, int upl, int nb) {
    return nb > 1 ? (upl > 1 ? 60 : 40) / (row_unit_words(wt) * upl * nw + nb * nw)
                  : 72 / (row_unit_words(wt) * upl * nw);
}
__host__ __device__ constexpr int row_batch(int wt, int nw, int upl, int nb) {
    return row_batch_raw(wt, nw, upl, nb) < 1 ? 1
         : row_batch_raw(wt, nw, upl, nb) > 32 / nb ? 32 / nb
         : row_batch_raw(wt, nw, upl, nb) > 4 ? 4
         : row_batch_raw(wt, nw, upl, nb);
}

// Shared memory of the kernel per x row: padded fp32 x, the int16 pairs
// (K/2 words), per-sub-block steps and sums (2 x K/32 floats).
__host__ __device__ constexpr size_t row_smem_bytes(int wt, int K) {
    return ((size_t)K + K / unit_weights(wt)) * 4 + (size_t)K / 2 * 4 + (size_t)K / 32 * 8;
}

// R1: one row per warp (matrices with too few rows to give every SM a
// CTA at the default row batch).
template <int WT, int EPI, int UPL, int NB, bool R1>
__global__ void __launch_bounds__(kRowThreads, 1) qgemv_row_kernel(QGemvArgs a, int nb) {
    constexpr int NW = EPI == kEpiSwiGLU ? 2 : 1;
    constexpr int UW = unit_weights(WT);
    constexpr int NSUB = UW / 32;
    constexpr int NWD = row_unit_words(WT);
    constexpr int R = R1 ? 1 : row_batch(WT, NW, UPL, NB);
    constexpr int U = UPL * kWarp;                      // units of a row
    constexpr int XQ = NSUB * 4 * U;                    // 16-byte chunks of one quantized x row
    extern __shared__ __align__(16) uint8_t smem[];
    const int XF = a.K + a.K / UW;                      // padded floats of one x row
    float *xs = reinterpret_cast<float *>(smem);                                 // [NB][XF]
    uint4 *xq4 = reinterpret_cast<uint4 *>(smem + (size_t)NB * XF * 4);          // [NB][sb][c][u]
    float *xst = reinterpret_cast<float *>(xq4 + (size_t)NB * XQ);               // [NB][sb][u] steps
    float *xsm = xst + NB * NSUB * U;                                            // [NB][sb][u] sums
    __shared__ float sred[NB][kRowThreads / kWarp];
    const int t = threadIdx.x, lane = t % kWarp, warp = t / kWarp;
    const size_t rb = a.plan.row_bytes;
    const int total = a.plan.total_rows;
    const int nwarps = (int)gridDim.x * (kRowThreads / kWarp);
    const int step = nwarps * R;
    int base = ((int)blockIdx.x * (kRowThreads / kWarp) + warp) * R;   // rows base .. base + R - 1

    uint32_t wq[R][NW][UPL][NWD];
    auto load_rows = [&](int b0) {
#pragma unroll
        for (int rr = 0; rr < R; ++rr) {
            int row = b0 + rr;
            if (row >= total) row = total - 1;           // loaded, never stored
            int m = 0, lr = row;
            while (m < a.n_seg - 1 && lr >= a.seg_rows[m]) lr -= a.seg_rows[m++];
#pragma unroll
            for (int w = 0; w < NW; ++w) {
                const uint8_t *src = reinterpret_cast<const uint8_t *>(a.W[w == 0 ? m : 1]) + (size_t)lr * rb;
#pragma unroll
                for (int i = 0; i < UPL; ++i) {
                    const uint32_t u = (uint32_t)(lane + kWarp * i);
                    if constexpr (WT == LI_WTYPE_Q8_0) {
                        const uint8_t *q = src + ((34u * u) & ~3u);
#pragma unroll
                        for (int k = 0; k < 9; ++k) wq[rr][w][i][k] = ldg_nc4(q + 4 * k);
                    } else {
                        const uint8_t *blk = src + 144 * (u >> 2);
                        const uint4 h = ldg_nc16(blk);
                        const uint4 qa = ldg_nc16(blk + 16 + 32 * (u & 3));
                        const uint4 qb = ldg_nc16(blk + 32 + 32 * (u & 3));
                        wq[rr][w][i][0] = h.x;  wq[rr][w][i][1] = h.y;  wq[rr][w][i][2] = h.z;  wq[rr][w][i][3] = h.w;
                        wq[rr][w][i][4] = qa.x; wq[rr][w][i][5] = qa.y; wq[rr][w][i][6] = qa.z; wq[rr][w][i][7] = qa.w;
                        wq[rr][w][i][8] = qb.x; wq[rr][w][i][9] = qb.y; wq[rr][w][i][10] = qb.z; wq[rr][w][i][11] = qb.w;
                    }
                }
            }
        }
    };
    // this lane's output: row base + lane / NB, x row lane % NB (lanes < R * NB)
    const int my_rr = lane / NB, my_b = lane % NB;
    const bool my_lane = lane < R * NB && my_b < nb;
    // in-projection epilogue inputs of this lane's output
    float c0 = 0.f, c1 = 0.f, c2 = 0.f;
    float4 cw = make_float4(0.f, 0.f, 0.f, 0.f);
    auto load_conv = [&](int b0) {
        if constexpr (EPI == kEpiConv) {
            const int row = b0 + my_rr;
            if (my_lane && row < total && row < a.conv_channels) {
                const float *cs = a.conv_state + ((size_t)my_b * a.conv_channels + row) * 3;
                c0 = cs[0]; c1 = cs[1]; c2 = cs[2];
                cw = *reinterpret_cast<const float4 *>(a.conv_w + 4 * (size_t)row);
            }
        }
    };

    if (base < total) load_rows(base);
    // x may be written by the previous kernel; a dependent launch may start
    // once that kernel has completed (the recurrence after a layer's first
    // GEMV reads its state before its own wait). The conv state read above
    // was last written by this layer's previous step, which had completed
    // before this kernel's predecessor could trigger it.
    grid_dep_wait();
    grid_dep_launch_dependents();
    {
        const float4 *g4 = reinterpret_cast<const float4 *>(a.gamma);
        float sq[NB];
#pragma unroll
        for (int b = 0; b < NB; ++b) {
            sq[b] = 0.f;
            if (b >= nb) continue;
            const float4 *x4 = reinterpret_cast<const float4 *>(a.x + (size_t)b * a.x_stride);
            for (int i = t; i < a.K / 4; i += kRowThreads) {
                float4 v = x4[i];
                sq[b] = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, sq[b]))));
                if (a.gamma) {
                    const float4 g = g4[i];
                    v.x *= g.x; v.y *= g.y; v.z *= g.z; v.w *= g.w;
                }
                const int k = 4 * i, kp = b * XF + k + k / UW;
                xs[kp] = v.x; xs[kp + 1] = v.y; xs[kp + 2] = v.z; xs[kp + 3] = v.w;
            }
        }
#pragma unroll
        for (int b = 0; b < NB; ++b) {
            const float v = warp_sum(sq[b]);
            if (lane == 0) sred[b][warp] = v;
        }
        __syncthreads();
        for (int q = t; q < nb * NSUB * U; q += kRowThreads) {   // q = (b * NSUB + sb) * U + u
            const int b = q / (NSUB * U), sb = (q / U) % NSUB, u = q % U;
            float rnorm = 1.0f;
            if (a.gamma) {
                float tot = 0.f;
                for (int w = 0; w < kRowThreads / kWarp; ++w) tot += sred[b][w];
                rnorm = rsqrtf(tot / (float)a.K + a.eps);
            }
            const float *xu = xs + (size_t)b * XF + (size_t)u * (UW + 1) + 32 * sb;
            float v[32];
            float sm = 0.f;
#pragma unroll
            for (int k = 0; k < 32; ++k) {
                v[k] = xu[k] * rnorm;
                sm += v[k];
            }
            int xq[16];
            xst[q] = quantize32_s16(v, xq);
            xsm[q] = sm;
#pragma unroll
            for (int c = 0; c < 4; ++c)
                xq4[(size_t)b * XQ + (size_t)(sb * 4 + c) * U + u] =
                    make_uint4(xq[4 * c], xq[4 * c + 1], xq[4 * c + 2], xq[4 * c + 3]);
        }
        __syncthreads();
    }
    load_conv(base);

    for (; base < total; base += step) {
        float acc[R][NW][NB];
#pragma unroll
        for (int rr = 0; rr < R; ++rr)
#pragma unroll
            for (int w = 0; w < NW; ++w)
#pragma unroll
                for (int b = 0; b < NB; ++b) acc[rr][w][b] = 0.f;
#pragma unroll
        for (int i = 0; i < UPL; ++i) {
            const int u = lane + kWarp * i;
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                if (b >= nb) break;
                int ia[R][NW][NSUB];
                float xsv[NSUB], xmv[NSUB];
#pragma unroll
                for (int sb = 0; sb < NSUB; ++sb) {
                    int xq[16];
                    const uint4 *xp = xq4 + (size_t)b * XQ + (size_t)sb * 4 * U + u;
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const uint4 v = xp[c * U];
                        xq[4 * c] = (int)v.x; xq[4 * c + 1] = (int)v.y; xq[4 * c + 2] = (int)v.z; xq[4 * c + 3] = (int)v.w;
                    }
                    xsv[sb] = xst[(b * NSUB + sb) * U + u];
                    xmv[sb] = xsm[(b * NSUB + sb) * U + u];
#pragma unroll
                    for (int rr = 0; rr < R; ++rr)
#pragma unroll
                        for (int w = 0; w < NW; ++w) {
                            if constexpr (WT == LI_WTYPE_Q8_0) {
                                acc[rr][w][b] += dot_q8_0_words(*reinterpret_cast<const uint32_t(*)[9]>(wq[rr][w][i]),
                                                                ((34u * (uint32_t)u) & 2u) != 0, xq, xsv[0]);
                            } else {
                                ia[rr][w][sb] = q4k_nibble_dot(*reinterpret_cast<const uint32_t(*)[8]>(wq[rr][w][i] + 4),
                                                               4u * (uint32_t)sb, xq);
                            }
                        }
                }
                if constexpr (WT == LI_WTYPE_Q4_K) {
#pragma unroll
                    for (int rr = 0; rr < R; ++rr)
#pragma unroll
                        for (int w = 0; w < NW; ++w) {
                            const uint32_t *v = wq[rr][w][i];
                            acc[rr][w][b] += q4k_combine(make_uint4(v[0], v[1], v[2], v[3]), u & 3, ia[rr][w][0],
                                                         ia[rr][w][NSUB - 1], xsv[0], xsv[NSUB - 1], xmv[0],
                                                         xmv[NSUB - 1]);
                        }
                }
            }
        }
        if (base + step < total) load_rows(base + step);
        float s0 = 0.f, s1 = 0.f;   // this lane's sums
#pragma unroll
        for (int rr = 0; rr < R; ++rr)
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                if (b >= nb) break;
                const float v0 = warp_sum(acc[rr][0][b]);
                const float v1 = NW == 2 ? warp_sum(acc[rr][NW - 1][b]) : 0.f;
                if (lane == rr * NB + b) { s0 = v0; s1 = v1; }
            }
        const int row = base + my_rr;
        if (my_lane && row < total) {
            if (EPI == kEpiSwiGLU) {
                a.dst[0][(size_t)my_b * a.dst_stride[0] + row] = silu(s0) * s1;
            } else if (EPI == kEpiStore) {
                int m = 0, lr = row;
                while (m < a.n_seg - 1 && lr >= a.seg_rows[m]) lr -= a.seg_rows[m++];
                float *d = m == 0 ? a.dst[0] : (m == 1 ? a.dst[1] : a.dst[2]);
                const int ds = m == 0 ? a.dst_stride[0] : (m == 1 ? a.dst_stride[1] : a.dst_stride[2]);
                float *o = d + (size_t)my_b * ds + lr;
                *o = a.accumulate ? *o + s0 : s0;
            } else {   // kEpiConv: DeltaNet in-projection epilogue
                float out = s0;
                if (row < a.conv_channels) {
                    float *cs = a.conv_state + ((size_t)my_b * a.conv_channels + row) * 3;
                    const float accv = fmaf(cw.x, c0, fmaf(cw.y, c1, fmaf(cw.z, c2, cw.w * s0)));
                    cs[0] = c1;
                    cs[1] = c2;
                    cs[2] = s0;
                    out = silu(accv);
                }
                a.dst[0][(size_t)my_b * a.dst_stride[0] + row] = out;
            }
        }
        load_conv(base + step);
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
    p->U = K / unit_weights(wtype);
    p->UP = (p->U + kWarp - 1) / kWarp * kWarp;
    if (p->UP > kMaxThreads) return LI_ERR_BAD_SHAPE;
    p->RP = p->UP >= 256 ? 1 : 256 / p->UP;
    const int nw = epi == kEpiSwiGLU ? 2 : 1;
    p->R = 8 / nw;
    while (p->R > 1 && (size_t)nw * p->RP * p->R * rb > kStageTarget) p->R >>= 1;
    p->SR = p->RP * p->R;
    p->row_bytes = rb;
    p->total_rows = total_rows;
    const size_t stage = (size_t)nw * p->SR * rb;
    p->S = (int)(kSmemBudget / stage);
    if (p->S > 4) p->S = 4;
    if (p->S < 2) p->S = 2;
    if (p->S * stage > 200 * 1024) return LI_ERR_BAD_SHAPE;
    // x staging (K floats + one pad per unit) borrows the first XB buffers
    const size_t xbytes = ((size_t)K + K / unit_weights(wtype)) * sizeof(float);
    p->XB = (int)((xbytes + stage - 1) / stage);
    if (p->S < p->XB + 1) p->S = p->XB + 1;
    if (p->S * stage > 200 * 1024) return LI_ERR_BAD_SHAPE;
    p->threads = p->UP * p->RP;
    p->smem = p->S * stage + p->S * sizeof(uint64_t) + 2 * (size_t)p->SR * (p->UP / kWarp) * nw * 4 + 16;
    return 0;
}

// Resident CTAs per SM of a kernel at (threads, smem). The kernel's dynamic
// shared-memory limit is raised to the device maximum once per (device,
// kernel), and the occupancy is cached per (device, kernel, threads, smem),
// so a launch makes no attribute or occupancy query after the first one
// (launches stay cheap and graph-capturable).
static int resident_ctas(const void *kern, int threads, size_t smem) {
    struct Entry { int dev; const void *k; int threads; size_t smem; int per_sm; };
    static std::mutex mu;
    static std::vector<Entry> cache;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    bool raised = false;
    for (const Entry &e : cache) {
        if (e.dev == dev && e.k == kern) {
            raised = true;
            if (e.threads == threads && e.smem == smem) return e.per_sm;
        }
    }
    cudaError_t e;
    if (!raised) {
        int max_optin = 0;
        e = cudaDeviceGetAttribute(&max_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        if (e != cudaSuccess) return -(int)e;
        cudaFuncAttributes fa;
        e = cudaFuncGetAttributes(&fa, kern);
        if (e != cudaSuccess) return -(int)e;
        // the limit covers dynamic shared memory only; static usage counts against the total
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 max_optin - (int)fa.sharedSizeBytes);
        if (e != cudaSuccess) return -(int)e;
    }
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, smem);
    if (e != cudaSuccess) return -(int)e;
    cache.push_back({dev, kern, threads, smem, per_sm});
    return per_sm;
}

template <int WT, int EPI, int R>
static const void *pick_kernel(int) {
    return (const void *)qgemv_kernel<WT, EPI, kMaxThreads, R>;
}

template <int WT, int EPI>
static int launch_t(const QGemvArgs &a, int n_rows, cudaStream_t stream, bool pdl) {
    const void *kern;
    switch (a.plan.R) {
    case 1: kern = pick_kernel<WT, EPI, 1>(a.plan.threads); break;
    case 2: kern = pick_kernel<WT, EPI, 2>(a.plan.threads); break;
    case 4: kern = pick_kernel<WT, EPI, 4>(a.plan.threads); break;
    default:
        if (EPI == kEpiSwiGLU) return LI_ERR_BAD_SHAPE;
        kern = pick_kernel<WT, EPI, EPI == kEpiSwiGLU ? 4 : 8>(a.plan.threads);
        break;
    }
    const int per_sm = resident_ctas(kern, a.plan.threads, a.plan.smem);
    if (per_sm < 0) return -per_sm;
    if (per_sm < 1) return LI_ERR_BAD_SHAPE;
    const int n_stages = (a.plan.total_rows + a.plan.SR - 1) / a.plan.SR;
    int grid = num_sms() * per_sm;
    if (grid > n_stages) grid = n_stages;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid, n_rows);
    cfg.blockDim = dim3(a.plan.threads);
    cfg.dynamicSmemBytes = a.plan.smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    void *params[] = {const_cast<QGemvArgs *>(&a)};
    return (int)cudaLaunchKernelExC(&cfg, kern, params);
}

// The few-row kernel: K a multiple of 32 units (every lane has UPL whole
// units), at most 4 units per lane for one x row (Q8_0) and 2 otherwise (x
// and the weights stay in registers), n_rows <= 8.
template <int WT, int EPI, int UPL, int NB, bool R1 = false>
static int launch_row_t(const QGemvArgs &a, int n_rows, cudaStream_t stream, bool pdl) {
    constexpr int R = R1 ? 1 : row_batch(WT, EPI == kEpiSwiGLU ? 2 : 1, UPL, NB);
    if constexpr (NB == 1 && !R1 && R > 1) {
        // groups of R rows per warp would leave more than half the SMs idle:
        // one row per warp (measured: the 3072-row Q8_0 QKV GEMV 9.8 -> 8.6 us;
        // at 58% of the SMs busy, the 4096-row out-projection, no gain)
        if (2 * a.plan.total_rows < kRowThreads / kWarp * R * num_sms())
            return launch_row_t<WT, EPI, UPL, NB, true>(a, n_rows, stream, pdl);
    }
    auto kern = qgemv_row_kernel<WT, EPI, UPL, NB, R1>;
    const size_t smem = NB * row_smem_bytes(WT, a.K);
    const int per_sm = resident_ctas((const void *)kern, kRowThreads, smem);
    if (per_sm < 0) return -per_sm;
    if (per_sm < 1) return LI_ERR_BAD_SHAPE;
    const int rows_per_cta = kRowThreads / kWarp * R;
    int grid = num_sms() * per_sm;
    const int need = (a.plan.total_rows + rows_per_cta - 1) / rows_per_cta;
    if (grid > need) grid = need;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kRowThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int nb = n_rows;
    void *params[] = {const_cast<QGemvArgs *>(&a), &nb};
    return (int)cudaLaunchKernelExC(&cfg, (const void *)kern, params);
}

template <int WT, int EPI, int UPL>
static int launch_row_nb(const QGemvArgs &a, int n_rows, cudaStream_t stream, bool pdl) {
    if (n_rows == 1) return launch_row_t<WT, EPI, UPL, 1>(a, n_rows, stream, pdl);
    if constexpr (UPL <= 2) {
        switch (n_rows) {
        case 2: return launch_row_t<WT, EPI, UPL, 2>(a, n_rows, stream, pdl);
        case 3: return launch_row_t<WT, EPI, UPL, 3>(a, n_rows, stream, pdl);
        case 4: return launch_row_t<WT, EPI, UPL, 4>(a, n_rows, stream, pdl);
        case 5:
        case 6: return launch_row_t<WT, EPI, UPL, 6>(a, n_rows, stream, pdl);
        default: return launch_row_t<WT, EPI, UPL, 8>(a, n_rows, stream, pdl);
        }
    }
    return LI_ERR_BAD_SHAPE;
}

template <int WT, int EPI>
static int launch_row(const QGemvArgs &a, int upl, int n_rows, cudaStream_t stream, bool pdl) {
    switch (upl) {
    case 1: return launch_row_nb<WT, EPI, 1>(a, n_rows, stream, pdl);
    case 2: return launch_row_nb<WT, EPI, 2>(a, n_rows, stream, pdl);
    default:
        if constexpr (WT == LI_WTYPE_Q8_0) {
            if (upl == 3) return launch_row_t<WT, EPI, 3, 1>(a, n_rows, stream, pdl);
            if (upl == 4) return launch_row_t<WT, EPI, 4, 1>(a, n_rows, stream, pdl);
        }
        return LI_ERR_BAD_SHAPE;
    }
}

// Units per lane of the few-row kernel for this shape, or 0 when it does not apply.
static int row_kernel_upl_shape(int wtype, int K, int n_rows) {
    if (n_rows < 1 || n_rows > kRowMaxBatch) return 0;
    if (wtype != LI_WTYPE_Q8_0 && wtype != LI_WTYPE_Q4_K) return 0;
    const int per_warp = unit_weights(wtype) * kWarp;
    if (K <= 0 || K % per_warp) return 0;
    const int upl = K / per_warp;
    const int max_upl = n_rows > 1 ? 2 : (wtype == LI_WTYPE_Q8_0 ? 4 : 2);
    return upl <= max_upl ? upl : 0;
}

static int row_kernel_upl(const QGemvArgs &a, int n_rows) {
    if (a.gamma && !aligned16(a.gamma)) return 0;
    if (!aligned16(a.x) || (n_rows > 1 && a.x_stride % 4)) return 0;
    return row_kernel_upl_shape(a.wtype, a.K, n_rows);
}

bool qgemv_few_rows(int wtype, int K, int n_rows) { return row_kernel_upl_shape(wtype, K, n_rows) != 0; }

int qgemv_launch(const QGemvArgs &a, int n_rows, cudaStream_t stream, bool pdl) {
    const int wt = a.wtype;
    if (const int upl = row_kernel_upl(a, n_rows)) {
        switch (a.epi) {
        case kEpiStore:
            return wt == LI_WTYPE_Q8_0 ? launch_row<LI_WTYPE_Q8_0, kEpiStore>(a, upl, n_rows, stream, pdl)
                                       : launch_row<LI_WTYPE_Q4_K, kEpiStore>(a, upl, n_rows, stream, pdl);
        case kEpiSwiGLU:
            return wt == LI_WTYPE_Q8_0 ? launch_row<LI_WTYPE_Q8_0, kEpiSwiGLU>(a, upl, n_rows, stream, pdl)
                                       : launch_row<LI_WTYPE_Q4_K, kEpiSwiGLU>(a, upl, n_rows, stream, pdl);
        case kEpiConv:
            return wt == LI_WTYPE_Q8_0 ? launch_row<LI_WTYPE_Q8_0, kEpiConv>(a, upl, n_rows, stream, pdl)
                                       : launch_row<LI_WTYPE_Q4_K, kEpiConv>(a, upl, n_rows, stream, pdl);
        default:
            return LI_ERR_BAD_ARG;
        }
    }
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
    if (!aligned16(W) || !aligned16(x)) return LI_ERR_MISALIGNED;   // x rows are read as float4
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
    if (gamma && !aligned16(gamma)) return LI_ERR_MISALIGNED;
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
    if (!aligned16(gamma)) return LI_ERR_MISALIGNED;
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

// Workspace regions, 256-byte aligned: h f32 [n_rows][N]; and for
// n_rows >= kTcMinRows (tensor-core path) also x16 f16 [n_rows][K],
// xscale [n_rows], h16 f16 [n_rows][N], hscale [n_rows], and the partial
// sums of the X-stationary projections (gate/up, then down, share them).
static size_t al256(size_t v) { return (v + 255) / 256 * 256; }

static size_t ffn_partials_bytes(int wtype, int K, int N, int n_rows) {
    const size_t pg = tc_gemm_partials_bytes(wtype, kTcSwiGLU, K, N, n_rows);
    const size_t pd = tc_gemm_partials_bytes(wtype, kTcStore, N, K, n_rows);
    return pg > pd ? pg : pd;
}

size_t li_fused_ffn_workspace_size(int K, int N, int n_rows) {
    if (K <= 0 || N <= 0 || n_rows <= 0) return 0;
    const size_t n = (size_t)n_rows;
    size_t b = al256((size_t)N * n * 4);
    const size_t nx = (n + 31) / 32 * 32;   // tiled X operands are padded to 32 rows
    if (n_rows >= kTcMinRows)
        b += al256((size_t)K * nx * 2) + al256(n * 4) + al256((size_t)N * nx * 2) + al256(n * 4) +
             al256(ffn_partials_bytes(LI_WTYPE_Q4_K, K, N, n_rows) > ffn_partials_bytes(LI_WTYPE_Q8_0, K, N, n_rows)
                       ? ffn_partials_bytes(LI_WTYPE_Q4_K, K, N, n_rows)
                       : ffn_partials_bytes(LI_WTYPE_Q8_0, K, N, n_rows));
    return b;
}

}  // extern "C"

// accumulate: y += ffn(x) (the down projection adds into y).
static int fused_ffn(int wtype, const float *x, const float *gamma, const void *Wg, const void *Wu, const void *Wd,
                     float *y, int K, int N, int n_rows, float eps, void *workspace, size_t workspace_bytes,
                     void *stream, bool accumulate) {
    int rc = common_q_checks(wtype, x, Wg, y, K, N, n_rows);
    if (!rc) rc = common_q_checks(wtype, x, Wu, y, K, N, n_rows);
    if (!rc) rc = common_q_checks(wtype, x, Wd, y, N, K, n_rows);
    if (rc) return rc;
    if (N == 0 || n_rows == 0) return 0;
    if (!workspace || workspace_bytes < li_fused_ffn_workspace_size(K, N, n_rows))
        return LI_ERR_WORKSPACE;
    if (gamma && !aligned16(gamma)) return LI_ERR_MISALIGNED;
    const cudaStream_t s = (cudaStream_t)stream;
    char *ws = (char *)workspace;
    float *h = (float *)ws;
    if (n_rows >= kTcMinRows && n_rows <= 256 && K % 256 == 0 && N % 256 == 0) {
        // tensor-core path: x -> f16, gate/up GEMM + SwiGLU, h -> f16, down GEMM
        const size_t n = (size_t)n_rows, nx = (n + 31) / 32 * 32;
        size_t off = al256((size_t)N * n * 4);
        __half *x16 = (__half *)(ws + off); off += al256((size_t)K * nx * 2);
        float *xs = (float *)(ws + off);    off += al256(n * 4);
        __half *h16 = (__half *)(ws + off); off += al256((size_t)N * nx * 2);
        float *hs = (float *)(ws + off);    off += al256(n * 4);
        float *partials = ffn_partials_bytes(wtype, K, N, n_rows) ? (float *)(ws + off) : nullptr;
        TcArgs d = {};
        d.wtype = wtype; d.epi = kTcStore; d.K = N; d.total_rows = K; d.B = n_rows;
        d.W[0] = Wd; d.n_seg = 1; d.seg_rows[0] = K; d.dst[0] = y; d.dst_stride[0] = K;
        d.X16 = h16; d.xscale = hs; d.partials = partials;
        d.accumulate = accumulate;
        d.x_npad = tc_gemm_x_npad(d);
        if (tc_gemm_splits_k(d) && !accumulate) {   // the down projection adds K-split partials into y
            const cudaError_t e = cudaMemsetAsync(y, 0, (size_t)n_rows * K * sizeof(float), s);
            if (e != cudaSuccess) return (int)e;
        }
        TcArgs g = {};
        g.wtype = wtype; g.epi = kTcSwiGLU; g.K = K; g.total_rows = N; g.B = n_rows;
        g.W[0] = Wg; g.W[1] = Wu; g.n_seg = 1; g.seg_rows[0] = N; g.dst[0] = h; g.dst_stride[0] = N;
        g.X16 = x16; g.xscale = xs; g.partials = partials;
        g.x_npad = tc_gemm_x_npad(g);
        if ((rc = tc_prep_launch(x, K, gamma, eps, n_rows, K, x16, xs, s, true, g.x_npad, tc_gemm_x_stationary(g))))
            return rc;
        if ((rc = tc_gemm_launch(g, s, true))) return rc;
        if ((rc = tc_prep_launch(h, N, nullptr, 0.f, n_rows, N, h16, hs, s, true, d.x_npad, tc_gemm_x_stationary(d))))
            return rc;
        return tc_gemm_launch(d, s, true);
    }
    QGemvArgs a = {};
    a.wtype = wtype; a.epi = kEpiSwiGLU;
    if ((rc = qgemv_plan(wtype, K, N, kEpiSwiGLU, &a.plan))) return rc;
    a.x = x; a.x_stride = K; a.gamma = gamma; a.K = K; a.eps = eps;
    a.n_seg = 1; a.W[0] = Wg; a.W[1] = Wu; a.seg_rows[0] = N;
    a.dst[0] = h; a.dst_stride[0] = N;
    // a plain launch: as a dependent launch (resident during the previous
    // down projection) the one-row FFN step measured 38.8 us against 30.7
    if ((rc = qgemv_launch(a, n_rows, s, false))) return rc;
    QGemvArgs dn = {};
    dn.wtype = wtype; dn.epi = kEpiStore;
    if ((rc = qgemv_plan(wtype, N, K, kEpiStore, &dn.plan))) return rc;
    dn.x = h; dn.x_stride = N; dn.gamma = nullptr; dn.K = N; dn.eps = 0.f;
    dn.n_seg = 1; dn.W[0] = Wd; dn.seg_rows[0] = K; dn.dst[0] = y; dn.dst_stride[0] = K;
    dn.accumulate = accumulate;
    return qgemv_launch(dn, n_rows, s, true);
}

extern "C" int li_launch_fused_ffn_q(int wtype, const float *x, const float *gamma, const void *Wg,
                                     const void *Wu, const void *Wd, float *y, int K, int N, int n_rows,
                                     float eps, void *workspace, size_t workspace_bytes, void *stream) {
    return fused_ffn(wtype, x, gamma, Wg, Wu, Wd, y, K, N, n_rows, eps, workspace, workspace_bytes, stream, false);
}

int li::fused_ffn_q_residual(int wtype, const float *x, const float *gamma, const void *Wg, const void *Wu,
                             const void *Wd, float *y, int K, int N, int n_rows, float eps, void *workspace,
                             size_t workspace_bytes, void *stream) {
    return fused_ffn(wtype, x, gamma, Wg, Wu, Wd, y, K, N, n_rows, eps, workspace, workspace_bytes, stream, true);
}
