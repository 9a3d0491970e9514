// Gated GQA attention layer, one decode step per sequence (the attention
// layers of the hybrid DeltaNet/attention stack; the reference describes them
// in docs/ASSESSMENT.md:1077 and :1086-1087 and has no kernel for them).
//
// Per sequence s, with the new token at position pos[s]:
//   p = W_in . rmsnorm?(x)                 rows q [Hq*D] | gate [Hq*D] | k [Hkv*D] | v [Hkv*D]
//   q_h = rope(rmsnorm(q_h) * q_norm_w),  k_j = rope(rmsnorm(k_j) * k_norm_w)
//   K[s][pos][j] = f16(k_j), V[s][pos][j] = f16(v_j)
//   o_h = softmax_t(q_h . K[s][t][j] / sqrt(D)) V[s][t][j],  t = 0..pos, j = h / (Hq/Hkv)
//   y = W_out . (o * sigmoid(gate))
//
// Kernels (one stream, programmatic dependent launches after the first):
//   projection     the quantized GEMV (SIMT, few rows) or the tcgen05 GEMM, as
//                  in the DeltaNet layer (li_qgemv.cu / li_tcgemm.cu);
//   attn_prep      one warp per (sequence, head): per-head RMSNorm and RoPE of
//                  q (in place, fp32) and k, k and v rounded to f16 into the
//                  caches at pos;
//   attn_decode    split-K decode attention: CTA (chunk, kv head, sequence)
//                  streams `chunk` cached tokens of one kv head once for all
//                  Hq/Hkv q heads of its group (K and V rows are read with
//                  16-byte loads, a half-warp per 256-byte row), online
//                  softmax per warp, the four warps merged in shared memory,
//                  and writes (max, sum, o[D]) per q head and chunk;
//   attn_combine   merges the chunks of each (sequence, head), divides by the
//                  softmax sum and applies sigmoid(gate);
//   out-projection the quantized GEMV or tcgen05 GEMM again.
// HBM-bound: a step reads each cached token's K and V row once per kv head.
#include "li_common.cuh"
#include "li_qgemv.cuh"
#include "li_tc.cuh"
#include "li_tcgemm.cuh"

#include <cuda.h>   // CUtensorMap and its enums; the encoder is fetched at run time

#include <cstring>
#include <mutex>

LI_DEFINE_TU_STATUS(attn)

namespace li {
namespace {

constexpr int kD = 128;              // head_dim (the only built size)
constexpr int kDecThreads = 128;     // 4 warps per attention CTA
constexpr int kSub = 16;             // tokens per warp per softmax sub-chunk (2 per iteration)
constexpr int kPartStride = kD + 4;  // floats per (sequence, head, chunk) record: m, l, pad, pad, o[D]

struct AttnArgs {
    float *proj;                 // [B][NP]: q | gate | k | v (q rewritten in place by attn_prep)
    int NP, Hq, Hkv, rope_dim;
    const float *q_norm_w, *k_norm_w;
    float eps;
    double log2_theta;
    const int *pos;              // [B]
    __half *k_cache, *v_cache;   // [B][max_ctx][Hkv][D]
    int max_ctx;
    int chunk, n_chunk;          // tokens per attention CTA, chunks per sequence (max)
    float *part;                 // [B][Hq][n_chunk][kPartStride]
    float *og;                   // [B][Hq*D] gated outputs (fp32)
    float scale;                 // D^-1/2
};

// ---------------------------------------------------------------------------
// attn_prep: warp per (sequence, head slot); slots 0..Hq-1 are q heads,
// Hq..Hq+Hkv-1 the kv heads (k normalised and rotated, v copied).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) attn_prep_kernel(AttnArgs a, int B) {
    __shared__ float vec[8][kD];
    grid_dep_wait();
    grid_dep_launch_dependents();
    const int wi = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
    const int slots = a.Hq + a.Hkv;
    const int gw = blockIdx.x * 8 + wi;
    if (gw >= B * slots) return;
    const int s = gw / slots, hs = gw % slots;
    const int pos = a.pos[s];
    if (pos < 0 || pos >= a.max_ctx) {
        // no cache slot for this token: nothing is written, the device flag is raised
        if (hs == 0 && lane == 0) atomicExch(&g_device_error, LI_ERR_BAD_ARG);
        return;
    }
    float *ps = a.proj + (size_t)s * a.NP;
    const bool is_q = hs < a.Hq;
    const int j = hs - a.Hq;
    float *src = is_q ? ps + (size_t)hs * kD : ps + (size_t)2 * a.Hq * kD + (size_t)j * kD;
    const float *w = is_q ? a.q_norm_w : a.k_norm_w;
    float v[4];
    float sq = 0.f;
#pragma unroll
    for (int m = 0; m < 4; ++m) {
        v[m] = src[lane + 32 * m];
        sq = fmaf(v[m], v[m], sq);
    }
    if (w) {
        const float r = rsqrtf(warp_sum(sq) / (float)kD + a.eps);
#pragma unroll
        for (int m = 0; m < 4; ++m) v[m] = v[m] * w[lane + 32 * m] * r;
    }
#pragma unroll
    for (int m = 0; m < 4; ++m) vec[wi][lane + 32 * m] = v[m];
    __syncwarp();
    const int half = a.rope_dim / 2;
#pragma unroll
    for (int m = 0; m < 4; ++m) {
        const int i = lane + 32 * m;
        if (i < a.rope_dim) {
            const int f = i < half ? i : i - half;   // frequency index
            // angle in double: pos * theta^(-2f/rope_dim) reaches ~pos radians
            const double ang = (double)pos * exp2(-(2.0 * f / a.rope_dim) * a.log2_theta);
            double sn, cs;
            sincos(ang, &sn, &cs);
            const float x1 = vec[wi][f], x2 = vec[wi][f + half];
            v[m] = i < half ? x1 * (float)cs - x2 * (float)sn : x2 * (float)cs + x1 * (float)sn;
        }
    }
    if (is_q) {
#pragma unroll
        for (int m = 0; m < 4; ++m) src[lane + 32 * m] = v[m];
    } else {
        const size_t off = (((size_t)s * a.max_ctx + pos) * a.Hkv + j) * kD;
        const float *vs = ps + (size_t)2 * a.Hq * kD + (size_t)a.Hkv * kD + (size_t)j * kD;
#pragma unroll
        for (int m = 0; m < 4; ++m) {
            a.k_cache[off + lane + 32 * m] = __float2half_rn(v[m]);
            a.v_cache[off + lane + 32 * m] = __float2half_rn(vs[lane + 32 * m]);
        }
    }
}

__device__ __forceinline__ void h8_to_f(const uint4 u, float (&f)[8]) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 t = __half22float2(*reinterpret_cast<const __half2 *>(&w[i]));
        f[2 * i] = t.x;
        f[2 * i + 1] = t.y;
    }
}

// 16 bytes global -> shared, asynchronous (zero-filled when !valid: a cache
// slot past the context may hold anything).
__device__ __forceinline__ void cp_async16(void *smem_dst, const void *gsrc, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(smem_dst)), "l"(gsrc),
                 "r"(valid ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Per warp and stage: the K and V rows of one sub-chunk, [K, V][kSub tokens][256 B].
constexpr int kStageBytes = 2 * kSub * kD * 2;
constexpr size_t kDecSmem = (size_t)4 * 2 * kStageBytes;   // 4 warps x 2 stages = 64 KB

// ---------------------------------------------------------------------------
// attn_decode: CTA (chunk, kv head j, sequence s), 4 warps. In a warp, lane
// l works on token (l / 16) of each pair of tokens and on dims 8*(l % 16) ..
// +7 of it; every q head of the group is held in registers for those dims.
// Each warp streams its tokens through two shared-memory stages with
// cp.async: the next sub-chunk's K and V rows are in flight while the current
// one is computed. A lane copies exactly the 16-byte pieces it reads later, so
// its own cp.async.wait_group is all the ordering it needs.
// ---------------------------------------------------------------------------
template <int G>
__global__ void __launch_bounds__(kDecThreads) attn_decode_kernel(AttnArgs a) {
    extern __shared__ __align__(16) uint8_t kv_smem[];   // [warp][stage][K, V][kSub][256 B]
    __shared__ float sc[4][G][kSub];                 // scores, then probabilities
    __shared__ float wm[4][G], wl[4][G];
    // each warp's partial o[G][D] for the merge, in its own staging area once
    // its loop is done (keeps the CTA at 65 KB of shared memory: 3 per SM)
    auto wo = [&](int w, int g) -> float * {
        return reinterpret_cast<float *>(kv_smem + (size_t)w * 2 * kStageBytes) + (size_t)g * kD;
    };
    grid_dep_wait();
    grid_dep_launch_dependents();
    const int chunk = blockIdx.x, j = blockIdx.y, s = blockIdx.z;
    const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
    const int hw = lane >> 4, c = lane & 15;
    const int pos = a.pos[s];
    const int t0 = chunk * a.chunk;
    const int t1 = min(min(t0 + a.chunk, pos + 1), a.max_ctx);   // a position past the cache reads none of it
    if (t0 >= t1 || pos < 0) return;                 // beyond this sequence's context
    // this warp's tokens: a contiguous quarter of the chunk's range
    const int per = (t1 - t0 + 3) / 4;
    const int wb = t0 + warp * per, we = min(wb + per, t1);

    float q[G][8];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        const float *qs = a.proj + (size_t)s * a.NP + (size_t)(j * G + g) * kD + 8 * c;
        const float4 q0 = *reinterpret_cast<const float4 *>(qs), q1 = *reinterpret_cast<const float4 *>(qs + 4);
        q[g][0] = q0.x * a.scale; q[g][1] = q0.y * a.scale; q[g][2] = q0.z * a.scale; q[g][3] = q0.w * a.scale;
        q[g][4] = q1.x * a.scale; q[g][5] = q1.y * a.scale; q[g][6] = q1.z * a.scale; q[g][7] = q1.w * a.scale;
    }
    float m[G], l[G], o[G][8];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.f;
#pragma unroll
        for (int d = 0; d < 8; ++d) o[g][d] = 0.f;
    }
    const size_t row_stride = (size_t)a.Hkv * kD;   // halves between consecutive tokens
    const __half *kbase = a.k_cache + ((size_t)s * a.max_ctx * a.Hkv + j) * kD + 8 * c;
    const __half *vbase = a.v_cache + ((size_t)s * a.max_ctx * a.Hkv + j) * kD + 8 * c;
    uint8_t *wbuf = kv_smem + (size_t)warp * 2 * kStageBytes;
    // this lane's 16-byte piece of row r of stage st: K at +0, V at +kSub*256
    auto piece = [&](int st, int r, int kv) -> uint8_t * {
        return wbuf + (size_t)st * kStageBytes + (size_t)kv * kSub * kD * 2 + (size_t)r * kD * 2 + 16 * c;
    };
    auto issue = [&](int tb, int st) {
#pragma unroll
        for (int it = 0; it < kSub / 2; ++it) {
            const int r = 2 * it + hw, t = tb + r;
            const bool ok = t < we;
            const size_t off = (size_t)(ok ? t : wb) * row_stride;
            cp_async16(piece(st, r, 0), kbase + off, ok);
            cp_async16(piece(st, r, 1), vbase + off, ok);
        }
        cp_async_commit();
    };
    if (wb < we) issue(wb, 0);

    int st = 0;
    for (int tb = wb; tb < we; tb += kSub, st ^= 1) {
        // the next sub-chunk goes in flight, then this one must have landed
        if (tb + kSub < we) {
            issue(tb + kSub, st ^ 1);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        // scores of kSub tokens (kSub/2 iterations of one token per half-warp)
#pragma unroll
        for (int it = 0; it < kSub / 2; ++it) {
            float kf[8];
            h8_to_f(*reinterpret_cast<const uint4 *>(piece(st, 2 * it + hw, 0)), kf);
            const int t = tb + 2 * it + hw;
#pragma unroll
            for (int g = 0; g < G; ++g) {
                float d = 0.f;
#pragma unroll
                for (int e = 0; e < 8; ++e) d = fmaf(q[g][e], kf[e], d);
#pragma unroll
                for (int off = 8; off > 0; off >>= 1) d += __shfl_xor_sync(0xffffffffu, d, off);
                if (c == g % 16) sc[warp][g][2 * it + hw] = t < we ? d : -INFINITY;
            }
        }
        __syncwarp();
        // online softmax over the sub-chunk: lane i (< kSub) owns token i
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const float sv = sc[warp][g][lane & (kSub - 1)];
            float cm = sv;
#pragma unroll
            for (int off = kSub / 2; off > 0; off >>= 1) cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, off));
            const float mn = fmaxf(m[g], cm);
            const float alpha = m[g] == -INFINITY ? 0.f : __expf(m[g] - mn);
            const float pv = sv == -INFINITY ? 0.f : __expf(sv - mn);
            float ps = pv;
#pragma unroll
            for (int off = kSub / 2; off > 0; off >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
            l[g] = l[g] * alpha + ps;
            m[g] = mn;
#pragma unroll
            for (int d = 0; d < 8; ++d) o[g][d] *= alpha;
            __syncwarp();
            if (lane < kSub) sc[warp][g][lane] = pv;
        }
        __syncwarp();
        // weighted V rows (zero-filled past the warp's range)
#pragma unroll
        for (int it = 0; it < kSub / 2; ++it) {
            float vf[8];
            h8_to_f(*reinterpret_cast<const uint4 *>(piece(st, 2 * it + hw, 1)), vf);
#pragma unroll
            for (int g = 0; g < G; ++g) {
                const float pw = sc[warp][g][2 * it + hw];
#pragma unroll
                for (int d = 0; d < 8; ++d) o[g][d] = fmaf(pw, vf[d], o[g][d]);
            }
        }
        __syncwarp();
    }
    // the two half-warps hold different tokens of the same running softmax
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int d = 0; d < 8; ++d) o[g][d] += __shfl_xor_sync(0xffffffffu, o[g][d], 16);
    __syncwarp();   // every lane of this warp is past its last read of the staging area
    if (lane < 16) {
#pragma unroll
        for (int g = 0; g < G; ++g) {
            *reinterpret_cast<float4 *>(wo(warp, g) + 8 * c) = make_float4(o[g][0], o[g][1], o[g][2], o[g][3]);
            *reinterpret_cast<float4 *>(wo(warp, g) + 8 * c + 4) = make_float4(o[g][4], o[g][5], o[g][6], o[g][7]);
        }
    }
    if (lane == 0) {
#pragma unroll
        for (int g = 0; g < G; ++g) { wm[warp][g] = m[g]; wl[warp][g] = l[g]; }
    }
    __syncthreads();
    // merge the 4 warps: thread d of the CTA owns dim d of every head
    const int d = threadIdx.x;
#pragma unroll
    for (int g = 0; g < G; ++g) {
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < 4; ++w) M = fmaxf(M, wm[w][g]);
        float L = 0.f, O = 0.f;
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            const float f = wm[w][g] == -INFINITY ? 0.f : __expf(wm[w][g] - M);
            L = fmaf(wl[w][g], f, L);
            O = fmaf(wo(w, g)[d], f, O);
        }
        float *rec = a.part + (((size_t)s * a.Hq + (size_t)j * G + g) * a.n_chunk + chunk) * kPartStride;
        rec[4 + d] = O;
        if (d == 0) { rec[0] = M; rec[1] = L; }
    }
}

// ---------------------------------------------------------------------------
// attn_decode on the tensor cores: a persistent CTA per SM walks the (chunk,
// kv head, sequence) items c, c + grid, ... with one continuous stream of
// 128-token K and V tiles (TMA, 32 KB each, a ring of four), so the copies of
// the next item are in flight while this one finishes. Per tile:
//   S^T[t][n] = K[t][:] . Qcat[n][:]   tcgen05, M = 128 tokens, N = 32, K = D:
//       Qcat rows 0..15 are the group's q heads rounded to f16 (hi), rows
//       16..31 the f16 remainders (lo), so hi + lo carries q to ~22 bits;
//   online softmax per head over the tile (warps 0-3, one token row each);
//   O^T[d][n] += V[:][d] . Pcat[n][:]  tcgen05, M = 128 dims (V read MN-major),
//       N = 32, K = 128 tokens, with Pcat = probabilities as f16 hi | lo;
// O is rescaled in tensor memory when a head's running max grows. Rows of the
// last tile past the sequence's position are masked (score -inf, V row zeroed
// in shared memory: a cache slot past the context may hold anything). The
// item's (max, sum, o[D]) per q head goes to the same records as the SIMT
// kernel's, merged by attn_combine.
// Warps: 0-3 softmax and epilogue, 4 TMA producer, 5 MMA issuer (and TMEM).
// ---------------------------------------------------------------------------
constexpr int kTcTok = 128;                        // tokens per K / V tile
constexpr int kTcRing = 4;                         // K and V tiles in flight
constexpr uint32_t kTcTileBytes = kTcTok * kD * 2; // 32 KB
constexpr uint32_t kTcOpBytes = 32 * kD * 2;       // Qcat / Pcat operand: 32 rows x 128 (8 KB)
constexpr uint32_t kTcOffQ = kTcRing * kTcTileBytes, kTcOffP = kTcOffQ + kTcOpBytes, kTcOffBar = kTcOffP + kTcOpBytes;
constexpr size_t kTcSmem = kTcOffBar + 256 + 1024;  // barriers, then slack for the 1 KB alignment
constexpr int kTcAttnThreads = 192;
constexpr uint32_t kIdescAMajorMN = 1u << 15;

__device__ __forceinline__ void tma_load_3d(void *smem_dst, const CUtensorMap *map, int x, int y, int z,
                                            uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4}], [%5];"
        ::"r"(smem_addr(smem_dst)), "l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar))
        : "memory");
}

// Named barrier 1 over the four softmax warps, returning whether any of them
// passed `v` (a timed-out wait), so that all four leave their loops together.
__device__ __forceinline__ bool softmax_bar_any(bool v) {
    uint32_t r;
    asm volatile("{\n\t.reg .pred pi, po;\n\tsetp.ne.u32 pi, %1, 0;\n\t"
                 "bar.red.or.pred po, 1, 128, pi;\n\tselp.u32 %0, 1, 0, po;\n\t}"
                 : "=r"(r) : "r"((uint32_t)v) : "memory");
    return r != 0;
}

__device__ __forceinline__ bool attn_wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (!mbar_wait(bar, parity)) {
        *abort_flag = 1;
        return false;
    }
    return true;
}

// Tokens [t0, t1) of an item and its tile count (0: past the context).
__device__ __forceinline__ int attn_item(const AttnArgs &a, int it, int &s, int &j, int &chunk, int &t0, int &t1) {
    chunk = it % a.n_chunk;
    j = (it / a.n_chunk) % a.Hkv;
    s = it / (a.n_chunk * a.Hkv);
    t0 = chunk * a.chunk;
    const int pos = a.pos[s];
    t1 = min(min(t0 + a.chunk, pos + 1), a.max_ctx);   // a position past the cache reads none of it
    return t0 < t1 && pos >= 0 ? (t1 - t0 + kTcTok - 1) / kTcTok : 0;
}

// byte offset of element (row, k) in a [32 rows][128] f16 operand (two 64-wide 128B-swizzled blocks)
__device__ __forceinline__ uint32_t op_off(int row, int k) {
    return (uint32_t)(k >> 6) * 4096u + sw128_off(row, (k & 63) >> 3) + (uint32_t)(k & 7) * 2u;
}

template <int G>
__global__ void __launch_bounds__(kTcAttnThreads, 1)
attn_decode_tc_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV, AttnArgs a,
                      int n_items) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    uint8_t *ring = smem, *qbuf = smem + kTcOffQ, *pbuf = smem + kTcOffP;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kTcOffBar);
    uint64_t *full = bars, *empty = bars + kTcRing;
    uint64_t *q_full = empty + kTcRing, *s_full = q_full + 1, *s_empty = s_full + 2, *p_full = s_empty + 2;
    uint64_t *pv_done = p_full + 1, *fin = pv_done + 1;
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(fin + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);
    __shared__ float red_m[4][16], red_s[4][16];
    const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp, tid = threadIdx.x;

    if (tid == 0) {
        for (int i = 0; i < kTcRing; ++i) { mbar_init(&full[i], 1); mbar_init(&empty[i], 1); }
        mbar_init(q_full, 4);
        for (int i = 0; i < 2; ++i) { mbar_init(&s_full[i], 1); mbar_init(&s_empty[i], 4); }
        mbar_init(p_full, 4);
        mbar_init(pv_done, 1);
        mbar_init(fin, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 5) tmem_alloc(tmem_holder, 128);
    if (warp < 4) {
        // the operands' padding rows (heads G..15 of each half) stay zero
        for (int i = tid; i < 2 * (int)kTcOpBytes / 16; i += 128)
            reinterpret_cast<uint4 *>(qbuf)[i] = make_uint4(0u, 0u, 0u, 0u);   // qbuf and pbuf are adjacent
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;
    grid_dep_wait();                 // q and the caches come from the previous kernels
    grid_dep_launch_dependents();

    if (warp == 4) {
        // ------------- producer: K_i, V_i of every item, in order -------------
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(&tmK) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(&tmV) : "memory");
            int n = 0;
            for (int it = blockIdx.x; it < n_items && !*abort_flag; it += gridDim.x) {
                int s, j, chunk, t0, t1;
                const int nt = attn_item(a, it, s, j, chunk, t0, t1);
                for (int i = 0; i < nt; ++i) {
                    const int z = s * a.max_ctx + t0 + i * kTcTok;
                    for (int kv = 0; kv < 2; ++kv, ++n) {
                        const int slot = n % kTcRing;
                        if (n >= kTcRing && !attn_wait(&empty[slot], (uint32_t)((n / kTcRing - 1) & 1), abort_flag))
                            break;
                        mbar_arrive_expect_tx(&full[slot], kTcTileBytes);
                        uint8_t *dst = ring + (size_t)slot * kTcTileBytes;
                        const CUtensorMap *m = kv ? &tmV : &tmK;
                        tma_load_3d(dst, m, 0, j, z, &full[slot]);
                        tma_load_3d(dst + kTcTileBytes / 2, m, 64, j, z, &full[slot]);
                    }
                }
            }
            // every copy issued has landed before the CTA exits
            for (int k = n - kTcRing < 0 ? 0 : n - kTcRing; k < n; ++k)
                mbar_wait(&full[k % kTcRing], (uint32_t)((k / kTcRing) & 1));
        }
    } else if (warp == 5) {
        // ------------- MMA issuer -------------
        if (lane == 0) {
            const uint32_t id_s = idesc_kf16(128, 32, false);
            const uint32_t id_pv = idesc_kf16(128, 32, false) | kIdescAMajorMN;
            int gt = 0, items = 0;
            bool ok = true;
            for (int it = blockIdx.x; ok && it < n_items; it += gridDim.x) {
                int s, j, chunk, t0, t1;
                const int nt = attn_item(a, it, s, j, chunk, t0, t1);
                if (nt == 0) continue;
                if (!(ok = attn_wait(q_full, (uint32_t)(items & 1), abort_flag))) break;
                ++items;
                // S for tile gt (ring slot of its K tile: 2*gt)
                auto issue_s = [&](int g) -> bool {
                    const int n = 2 * g, slot = n % kTcRing, b = g & 1;
                    if (!attn_wait(&full[slot], (uint32_t)((n / kTcRing) & 1), abort_flag)) return false;
                    if (g >= 2 && !attn_wait(&s_empty[b], (uint32_t)(((g >> 1) - 1) & 1), abort_flag)) return false;
                    tc_fence_after();
                    const uint32_t kb = smem_addr(ring + (size_t)slot * kTcTileBytes);
                    for (int kk = 0; kk < 8; ++kk) {
                        const uint64_t ad = sw128_desc(kb + (uint32_t)(kk >> 2) * 16384u) + 2 * (kk & 3);
                        const uint64_t bd = sw128_desc(smem_addr(qbuf) + (uint32_t)(kk >> 2) * 4096u) + 2 * (kk & 3);
                        umma_f16(tmem + 32u * b, ad, bd, id_s, kk ? 1u : 0u);
                    }
                    umma_commit(&s_full[b]);
                    umma_commit(&empty[slot]);
                    return true;
                };
                if (!(ok = issue_s(gt))) break;
                for (int i = 0; i < nt; ++i) {
                    if (i + 1 < nt && !(ok = issue_s(gt + 1))) break;
                    // O^T += V^T Pcat for tile gt (ring slot of its V tile: 2*gt+1)
                    const int n = 2 * gt + 1, slot = n % kTcRing;
                    if (!(ok = attn_wait(&full[slot], (uint32_t)((n / kTcRing) & 1), abort_flag))) break;
                    if (!(ok = attn_wait(p_full, (uint32_t)(gt & 1), abort_flag))) break;
                    tc_fence_after();
                    const uint32_t vb = smem_addr(ring + (size_t)slot * kTcTileBytes);
                    for (int kk = 0; kk < 8; ++kk) {
                        const uint64_t ad = sw128_mn_desc(vb + (uint32_t)kk * 2048u, 16384u);
                        const uint64_t bd = sw128_desc(smem_addr(pbuf) + (uint32_t)(kk >> 2) * 4096u) + 2 * (kk & 3);
                        umma_f16(tmem + 64u, ad, bd, id_pv, (i | kk) ? 1u : 0u);
                    }
                    umma_commit(pv_done);
                    umma_commit(&empty[slot]);
                    ++gt;
                }
            }
            // every MMA issued has completed before the tensor memory is freed
            umma_commit(fin);
            mbar_wait(fin, 0u);
        }
    } else {
        // ------------- softmax (thread = token row of S^T, dim row of O^T) -------------
        // A timed-out wait never leaves a loop by itself: the warp carries on
        // (its later waits return at once) to the next named barrier, which
        // tells all four warps to stop.
        const uint32_t lane_base = tmem + ((uint32_t)(32 * warp) << 16);
        int gt = 0;
        bool stop = false;
        for (int it = blockIdx.x; !stop && it < n_items; it += gridDim.x) {
            int s, j, chunk, t0, t1;
            const int nt = attn_item(a, it, s, j, chunk, t0, t1);
            if (nt == 0) continue;
            // Qcat for this item (the previous item's S products have completed: their results were read)
            {
                const float *qs = a.proj + (size_t)s * a.NP + (size_t)j * G * kD + tid;
#pragma unroll
                for (int h = 0; h < G; ++h) {
                    const float q = qs[(size_t)h * kD] * a.scale;
                    const __half hi = __float2half_rn(q);
                    *reinterpret_cast<__half *>(qbuf + op_off(h, tid)) = hi;
                    *reinterpret_cast<__half *>(qbuf + op_off(16 + h, tid)) = __float2half_rn(q - __half2float(hi));
                }
            }
            fence_proxy_async_shared();
            __syncwarp();
            if (lane == 0) mbar_arrive(q_full);
            float m[G], l[G];
#pragma unroll
            for (int h = 0; h < G; ++h) { m[h] = -INFINITY; l[h] = 0.f; }
            for (int i = 0; i < nt; ++i, ++gt) {
                const int b = gt & 1;
                const bool w_ok = __all_sync(0xffffffffu, attn_wait(&s_full[b], (uint32_t)((gt >> 1) & 1), abort_flag));
                uint32_t sv[32];
                if (w_ok) {
                    tc_fence_after();
                    tmem_ld32_nowait(lane_base + 32u * b, sv);
                    tmem_wait_ld();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&s_empty[b]);
                }
                const bool valid = w_ok && t0 + i * kTcTok + tid < t1;
                float sc[G], p[G];
#pragma unroll
                for (int h = 0; h < G; ++h) {
                    sc[h] = valid ? __uint_as_float(sv[h]) + __uint_as_float(sv[16 + h]) : -INFINITY;
                    float mx = sc[h];
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
                    if (lane == 0) red_m[warp][h] = mx;
                }
                if ((stop = softmax_bar_any(!w_ok))) break;
                float alpha[G];
                bool grow = false;
#pragma unroll
                for (int h = 0; h < G; ++h) {
                    const float tm = fmaxf(fmaxf(red_m[0][h], red_m[1][h]), fmaxf(red_m[2][h], red_m[3][h]));
                    const float mn = fmaxf(m[h], tm);          // finite: the tile holds a valid token
                    alpha[h] = m[h] == -INFINITY ? 0.f : __expf(m[h] - mn);
                    grow |= m[h] != mn;
                    m[h] = mn;
                    p[h] = valid ? __expf(sc[h] - mn) : 0.f;
                    float ps = p[h];
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
                    if (lane == 0) red_s[warp][h] = ps;
                }
                asm volatile("bar.sync 1, 128;" ::: "memory");
#pragma unroll
                for (int h = 0; h < G; ++h)
                    l[h] = l[h] * alpha[h] + ((red_s[0][h] + red_s[1][h]) + (red_s[2][h] + red_s[3][h]));
                // the previous tile's O product has finished: Pcat may be rewritten, O rescaled
                bool ok2 = i == 0 || __all_sync(0xffffffffu, attn_wait(pv_done, (uint32_t)((gt - 1) & 1), abort_flag));
                // this tile's V has landed: rows past the context are zeroed (their products with p = 0 must be 0)
                const int n = 2 * gt + 1, slot = n % kTcRing;
                ok2 = ok2 && __all_sync(0xffffffffu, attn_wait(&full[slot], (uint32_t)((n / kTcRing) & 1), abort_flag));
                if (!ok2) continue;                   // the next tile's barrier stops every warp
                tc_fence_after();
                if (i > 0 && grow) {
                    uint32_t ov[32];
                    tmem_ld32_nowait(lane_base + 64u, ov);
                    tmem_wait_ld();
#pragma unroll
                    for (int h = 0; h < G; ++h) {
                        ov[h] = __float_as_uint(__uint_as_float(ov[h]) * alpha[h]);
                        ov[16 + h] = __float_as_uint(__uint_as_float(ov[16 + h]) * alpha[h]);
                    }
                    tmem_st32(lane_base + 64u, ov);
                    tmem_wait_st();
                }
#pragma unroll
                for (int h = 0; h < G; ++h) {
                    const __half hi = __float2half_rn(p[h]);
                    *reinterpret_cast<__half *>(pbuf + op_off(h, tid)) = hi;
                    *reinterpret_cast<__half *>(pbuf + op_off(16 + h, tid)) = __float2half_rn(p[h] - __half2float(hi));
                }
                if (t0 + i * kTcTok + tid >= t1) {
                    uint8_t *vrow = ring + (size_t)slot * kTcTileBytes + (size_t)tid * 128;
#pragma unroll
                    for (int q16 = 0; q16 < 8; ++q16) {
                        reinterpret_cast<uint4 *>(vrow)[q16] = make_uint4(0u, 0u, 0u, 0u);
                        reinterpret_cast<uint4 *>(vrow + kTcTileBytes / 2)[q16] = make_uint4(0u, 0u, 0u, 0u);
                    }
                }
                fence_proxy_async_shared();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(p_full);
            }
            if (stop) break;
            // the item's last O product, then its records
            if (!__all_sync(0xffffffffu, attn_wait(pv_done, (uint32_t)((gt - 1) & 1), abort_flag))) continue;
            tc_fence_after();
            uint32_t ov[32];
            tmem_ld32_nowait(lane_base + 64u, ov);
            tmem_wait_ld();
            tc_fence_before();
#pragma unroll
            for (int h = 0; h < G; ++h) {
                float *rec = a.part + (((size_t)s * a.Hq + (size_t)j * G + h) * a.n_chunk + chunk) * kPartStride;
                rec[4 + tid] = __uint_as_float(ov[h]) + __uint_as_float(ov[16 + h]);
                if (tid == 0) { rec[0] = m[h]; rec[1] = l[h]; }
            }
        }
    }

    if (*abort_flag && tid == 0) atomicExch(&g_device_error, LI_ERR_TIMEOUT);
    tc_fence_before();
    __syncthreads();
    if (warp == 5) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, 128);
    }
}

// ---------------------------------------------------------------------------
// attn_combine: CTA per (sequence, head), thread per dim.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kD) attn_combine_kernel(AttnArgs a) {
    grid_dep_wait();
    grid_dep_launch_dependents();
    const int s = blockIdx.x / a.Hq, h = blockIdx.x % a.Hq, d = threadIdx.x;
    const int pos = a.pos[s];
    if (pos < 0 || pos >= a.max_ctx) {                 // no context (the prep raised the device flag)
        a.og[(size_t)s * a.Hq * kD + (size_t)h * kD + d] = 0.f;
        return;
    }
    const int nch = (pos + a.chunk) / a.chunk;         // chunks holding tokens 0..pos
    const float *rec = a.part + ((size_t)s * a.Hq + h) * a.n_chunk * kPartStride;
    float M = -INFINITY;
    for (int c = 0; c < nch; ++c) M = fmaxf(M, rec[(size_t)c * kPartStride]);
    float L = 0.f, O = 0.f;
    for (int c = 0; c < nch; ++c) {
        const float *r = rec + (size_t)c * kPartStride;
        const float f = __expf(r[0] - M);
        L = fmaf(r[1], f, L);
        O = fmaf(r[4 + d], f, O);
    }
    const float gate = a.proj[(size_t)s * a.NP + (size_t)a.Hq * kD + (size_t)h * kD + d];
    a.og[(size_t)s * a.Hq * kD + (size_t)h * kD + d] = O / L * sigmoid(gate);
}

template <int G>
int launch_decode(const AttnArgs &a, int B, cudaStream_t s) {
    static std::once_flag once;
    static cudaError_t attr_err = cudaSuccess;
    std::call_once(once, [] {
        attr_err = cudaFuncSetAttribute(attn_decode_kernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)kDecSmem);
    });
    if (attr_err != cudaSuccess) return (int)attr_err;
    return (int)launch_pdl(attn_decode_kernel<G>, dim3((unsigned)a.n_chunk, (unsigned)a.Hkv, (unsigned)B),
                           dim3(kDecThreads), kDecSmem, s, true, a);
}

int launch_decode_any(int G, const AttnArgs &a, int B, cudaStream_t s) {
    switch (G) {
    case 1: return launch_decode<1>(a, B, s);
    case 2: return launch_decode<2>(a, B, s);
    case 3: return launch_decode<3>(a, B, s);
    case 4: return launch_decode<4>(a, B, s);
    case 5: return launch_decode<5>(a, B, s);
    case 6: return launch_decode<6>(a, B, s);
    case 8: return launch_decode<8>(a, B, s);
    default: return LI_ERR_UNSUPPORTED;
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

// A cache [B][max_ctx][Hkv][128] f16 as a 3-D tensor (d, kv head, B*max_ctx
// token rows) with a [128 tokens][1][64 d] box, 128-byte swizzle (rows past
// the last sequence's slots come in as zeros).
int encode_cache(CUtensorMap *m, void *base, int Hkv, long long rows) {
    EncodeTiledFn fn = encoder();
    if (!fn) return LI_ERR_UNSUPPORTED;
    const cuuint64_t dims[3] = {(cuuint64_t)kD, (cuuint64_t)Hkv, (cuuint64_t)rows};
    const cuuint64_t strides[2] = {(cuuint64_t)kD * 2, (cuuint64_t)Hkv * kD * 2};
    const cuuint32_t box[3] = {64, 1, (cuuint32_t)kTcTok};
    const cuuint32_t estr[3] = {1, 1, 1};
    const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, base, dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : LI_ERR_BAD_SHAPE;
}

// The tensor-core decode kernel where it applies: whole 128-token tiles per
// chunk, and the group's q heads in one half of the 32 MMA columns.
bool attn_tc(int G, int chunk) { return chunk % kTcTok == 0 && G >= 1 && G <= 16; }

template <int G>
int launch_decode_tc(const AttnArgs &a, int B, cudaStream_t s) {
    static std::once_flag once;
    static cudaError_t attr_err = cudaSuccess;
    std::call_once(once, [] {
        attr_err = cudaFuncSetAttribute(attn_decode_tc_kernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)kTcSmem);
    });
    if (attr_err != cudaSuccess) return (int)attr_err;
    CUtensorMap mk, mv;
    memset(&mk, 0, sizeof(mk));
    memset(&mv, 0, sizeof(mv));
    const long long rows = (long long)B * a.max_ctx;
    if (rows + kTcTok >= (1ll << 31)) return LI_ERR_BAD_SHAPE;
    int rc;
    if ((rc = encode_cache(&mk, a.k_cache, a.Hkv, rows)) || (rc = encode_cache(&mv, a.v_cache, a.Hkv, rows))) return rc;
    const int items = a.n_chunk * a.Hkv * B;
    const int grid = items < num_sms() ? items : num_sms();
    return (int)launch_pdl(attn_decode_tc_kernel<G>, dim3((unsigned)grid), dim3(kTcAttnThreads), kTcSmem, s, true,
                           mk, mv, a, items);
}

int launch_decode_tc_any(int G, const AttnArgs &a, int B, cudaStream_t s) {
    switch (G) {
    case 1: return launch_decode_tc<1>(a, B, s);
    case 2: return launch_decode_tc<2>(a, B, s);
    case 3: return launch_decode_tc<3>(a, B, s);
    case 4: return launch_decode_tc<4>(a, B, s);
    case 5: return launch_decode_tc<5>(a, B, s);
    case 6: return launch_decode_tc<6>(a, B, s);
    case 8: return launch_decode_tc<8>(a, B, s);
    default: return LI_ERR_UNSUPPORTED;
    }
}

size_t al256(size_t v) { return (v + 255) / 256 * 256; }

// Tokens per attention CTA: enough CTAs to cover the SMs several times over
// (about 2048), at least 64 (four warps of one sub-chunk each), at most 1024.
int pick_chunk(int B, int Hkv, int max_ctx) {
    const long long want = (long long)B * Hkv * max_ctx / 2048;
    int c = 64;
    while (c < 1024 && c < want) c <<= 1;
    return c;
}

// Projections on the SIMT GEMVs below kTcMinRows rows, and up to 3 rows when
// both shapes suit the few-row kernel; on the tensor cores otherwise (the
// rule of the DeltaNet layer).
bool attn_simt(const li_attn_layer *L, int n) {
    if (n < kTcMinRows) return true;
    return n <= 3 && qgemv_few_rows(L->w_in_type, L->hidden, n) &&
           qgemv_few_rows(L->w_out_type, L->n_q_heads * L->head_dim, n);
}

struct AttnWs {
    size_t proj, part, og, x16, xscale, og16, oscale, partials, total;
};

AttnWs attn_ws_layout(const li_attn_layer *L, int n, int max_ctx) {
    AttnWs w = {};
    const size_t D = L->head_dim, Hq = L->n_q_heads, Hkv = L->n_kv_heads, nn = (size_t)n;
    const size_t NP = 2 * Hq * D + 2 * Hkv * D;
    const int chunk = pick_chunk(n, (int)Hkv, max_ctx);
    const size_t nch = ((size_t)max_ctx + chunk - 1) / chunk;
    size_t off = 0;
    w.proj = off; off += al256(NP * nn * 4);
    w.part = off; off += al256(nn * Hq * nch * kPartStride * 4);
    w.og = off; off += al256(Hq * D * nn * 4);
    if (!attn_simt(L, n)) {
        const size_t nx = (nn + 31) / 32 * 32;
        w.x16 = off; off += al256((size_t)L->hidden * nx * 2);
        w.xscale = off; off += al256(nn * 4);
        w.og16 = off; off += al256(Hq * D * nx * 2);
        w.oscale = off; off += al256(nn * 4);
        const size_t pin = tc_gemm_partials_bytes(L->w_in_type, kTcStore, L->hidden, (int)NP, n);
        const size_t pout = tc_gemm_partials_bytes(L->w_out_type, kTcStore, (int)(Hq * D), L->hidden, n);
        w.partials = off; off += al256(pin > pout ? pin : pout);
    }
    w.total = off;
    return w;
}

// One projection y[b] = W . (rmsnorm?(x[b])): SIMT GEMV or prep + tcgen05 GEMM;
// accumulate: y[b] += W . x[b] (a residual update of dst).
int project(bool simt, int wtype, const void *W, int K, int N, const float *x, const float *gamma, float eps,
            float *dst, int B, char *ws, const AttnWs &lay, bool first, bool out, cudaStream_t s,
            bool accumulate = false) {
    int rc;
    if (simt) {
        QGemvArgs g = {};
        g.wtype = wtype; g.epi = kEpiStore;
        if ((rc = qgemv_plan(wtype, K, N, kEpiStore, &g.plan))) return rc;
        g.x = x; g.x_stride = K; g.gamma = gamma; g.K = K; g.eps = eps;
        g.n_seg = 1; g.W[0] = W; g.seg_rows[0] = N; g.dst[0] = dst; g.dst_stride[0] = N;
        g.accumulate = accumulate;
        return qgemv_launch(g, B, s, !first);
    }
    TcArgs t = {};
    t.wtype = wtype; t.epi = kTcStore; t.K = K; t.total_rows = N; t.B = B;
    t.W[0] = W; t.n_seg = 1; t.seg_rows[0] = N; t.dst[0] = dst; t.dst_stride[0] = N;
    t.X16 = reinterpret_cast<const __half *>(ws + (out ? lay.og16 : lay.x16));
    t.xscale = reinterpret_cast<const float *>(ws + (out ? lay.oscale : lay.xscale));
    t.partials = lay.partials ? reinterpret_cast<float *>(ws + lay.partials) : nullptr;
    t.accumulate = accumulate;
    t.x_npad = tc_gemm_x_npad(t);
    // a dependent launch also as the layer's first kernel: the prep waits for the previous kernel before it reads x
    if ((rc = tc_prep_launch(x, K, gamma, eps, B, K, const_cast<__half *>(t.X16), const_cast<float *>(t.xscale), s,
                             true, t.x_npad, tc_gemm_x_stationary(t))))
        return rc;
    if (tc_gemm_splits_k(t) && !accumulate) {
        // the K-split CTAs add into dst; ordered after the prep by the stream
        cudaError_t e = cudaMemsetAsync(dst, 0, (size_t)B * N * sizeof(float), s);
        if (e != cudaSuccess) return (int)e;
        return tc_gemm_launch(t, s, false);
    }
    return tc_gemm_launch(t, s, true);
}

}  // namespace
}  // namespace li

using namespace li;

extern "C" {

size_t li_attn_layer_workspace_size(const li_attn_layer *L, int n_seqs, int max_ctx) {
    if (!L || n_seqs <= 0 || max_ctx <= 0 || L->n_kv_heads <= 0 || L->head_dim != kD) return 0;
    return attn_ws_layout(L, n_seqs, max_ctx).total;
}

}  // extern "C"

// accumulate: y += the layer's output (the output projection adds into y).
static int attn_layer_decode(const li_attn_layer *L, const float *x, float *y, void *k_cache, void *v_cache,
                             const int32_t *pos, int n_seqs, int max_ctx, void *workspace, size_t workspace_bytes,
                             void *stream, bool accumulate) {
    if (!L || !x || !y || !k_cache || !v_cache || !pos || n_seqs < 0 || max_ctx <= 0) return LI_ERR_BAD_ARG;
    if (n_seqs == 0) return 0;
    if (!L->w_in || !L->w_out) return LI_ERR_BAD_ARG;
    if (L->head_dim != kD) return LI_ERR_UNSUPPORTED;
    const int Hq = L->n_q_heads, Hkv = L->n_kv_heads;
    if (Hkv <= 0 || Hq <= 0 || Hq % Hkv) return LI_ERR_BAD_SHAPE;
    const int G = Hq / Hkv;
    if (G > 8 || G == 7) return LI_ERR_UNSUPPORTED;
    if (L->rope_dim < 0 || L->rope_dim % 2 || L->rope_dim > kD) return LI_ERR_BAD_SHAPE;
    if (L->rope_dim > 0 && !(L->rope_theta > 1.0f)) return LI_ERR_BAD_ARG;
    if ((L->w_in_type != LI_WTYPE_Q4_K && L->w_in_type != LI_WTYPE_Q8_0) ||
        (L->w_out_type != LI_WTYPE_Q4_K && L->w_out_type != LI_WTYPE_Q8_0))
        return LI_ERR_UNSUPPORTED;
    if (!aligned16(x) || !aligned16(y) || !aligned16(k_cache) || !aligned16(v_cache)) return LI_ERR_MISALIGNED;
    if (L->in_norm_w && !aligned16(L->in_norm_w)) return LI_ERR_MISALIGNED;
    const AttnWs lay = attn_ws_layout(L, n_seqs, max_ctx);
    if (!workspace || workspace_bytes < lay.total) return LI_ERR_WORKSPACE;
    if (!aligned16(workspace)) return LI_ERR_MISALIGNED;
    char *ws = (char *)workspace;
    const cudaStream_t s = (cudaStream_t)stream;
    const int D = kD, NP = 2 * Hq * D + 2 * Hkv * D;
    const bool simt = attn_simt(L, n_seqs);
    int rc;

    AttnArgs a = {};
    a.proj = reinterpret_cast<float *>(ws + lay.proj);
    a.NP = NP; a.Hq = Hq; a.Hkv = Hkv; a.rope_dim = L->rope_dim;
    a.q_norm_w = L->q_norm_w; a.k_norm_w = L->k_norm_w; a.eps = L->qk_norm_eps;
    a.log2_theta = L->rope_dim > 0 ? log2((double)L->rope_theta) : 0.0;
    a.pos = pos;
    a.k_cache = static_cast<__half *>(k_cache); a.v_cache = static_cast<__half *>(v_cache);
    a.max_ctx = max_ctx;
    a.chunk = pick_chunk(n_seqs, Hkv, max_ctx);
    a.n_chunk = (max_ctx + a.chunk - 1) / a.chunk;
    a.part = reinterpret_cast<float *>(ws + lay.part);
    a.og = reinterpret_cast<float *>(ws + lay.og);
    a.scale = 1.0f / sqrtf((float)D);

    // 1. input projection (RMSNorm fused): a plain launch on the few-row path;
    //    on the tensor-core path its x prep is a dependent launch that waits
    //    for the previous kernel before it reads x
    if ((rc = project(simt, L->w_in_type, L->w_in, L->hidden, NP, x, L->in_norm_w, L->in_norm_eps, a.proj, n_seqs,
                      ws, lay, true, false, s)))
        return rc;
    // 2. per-head norm + RoPE, cache append
    const int warps = n_seqs * (Hq + Hkv);
    if ((rc = (int)launch_pdl(attn_prep_kernel, dim3((unsigned)((warps + 7) / 8)), dim3(256), 0, s, true, a,
                              n_seqs)))
        return rc;
    // 3. split-K attention (tensor cores for whole 128-token tiles), 4. merge + output gate
    if ((rc = attn_tc(G, a.chunk) ? launch_decode_tc_any(G, a, n_seqs, s) : launch_decode_any(G, a, n_seqs, s)))
        return rc;
    if ((rc = (int)launch_pdl(attn_combine_kernel, dim3((unsigned)(n_seqs * Hq)), dim3(kD), 0, s, true, a)))
        return rc;
    // 5. output projection
    return project(simt, L->w_out_type, L->w_out, Hq * D, L->hidden, a.og, nullptr, 0.f, y, n_seqs, ws, lay, false,
                   true, s, accumulate);
}

extern "C" int li_launch_attn_layer_decode(const li_attn_layer *L, const float *x, float *y, void *k_cache,
                                           void *v_cache, const int32_t *pos, int n_seqs, int max_ctx,
                                           void *workspace, size_t workspace_bytes, void *stream) {
    return attn_layer_decode(L, x, y, k_cache, v_cache, pos, n_seqs, max_ctx, workspace, workspace_bytes, stream,
                             false);
}

int li::attn_layer_decode_residual(const li_attn_layer *L, const float *x, float *y, void *k_cache, void *v_cache,
                                   const int32_t *pos, int n_seqs, int max_ctx, void *workspace,
                                   size_t workspace_bytes, void *stream) {
    return attn_layer_decode(L, x, y, k_cache, v_cache, pos, n_seqs, max_ctx, workspace, workspace_bytes, stream,
                             true);
}
