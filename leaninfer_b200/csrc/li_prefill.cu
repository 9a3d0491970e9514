// Chunked (WY form, chunk 64) gated delta rule prefill on the tensor cores.
//
// Semantics (per v-head h, k-head hk = h / (Hv/Hk), tokens t = 0..T-1):
//   a_t = exp(g_t); q~_t = scale * q_t;
//   v'_t = beta_t * (v_t - a_t * S^T k_t);  S <- a_t * S + k_t v'_t^T;  o_t = S^T q~_t
// with S[k][v] fp32 (the oracle's token-by-token restatement, lio_gdr_prefill).
// Over a chunk of C = 64 tokens with gamma_i = prod_{j<=i} a_j (computed as
// exp of a prefix sum of g) the chunk is exactly
//   A[i][j] = beta_i (gamma_i/gamma_j) k_i.k_j  (j < i),   T = (I + A)^-1,
//   W = T diag(beta gamma) K,   U = T diag(beta) V,   Delta = U - W S0,
//   P[i][j] = (gamma_i/gamma_j) q~_i.k_j (j <= i),
//   O = diag(gamma) Q~ S0 + P Delta,   S = gamma_C S0 + K^T diag(gamma_C/gamma) Delta.
//
// Two kernels:
//   gdr_prep_kernel (one CTA per v-head and pair of chunks, all in parallel):
//     K, Q, V rows of the 128-token pair by TMA, K K^T and Q K^T on tcgen05
//     (M = 128; the diagonal 64x64 blocks are the chunks'), A and P from them,
//     T by fp32 forward substitution (one column per thread, in registers), W
//     and U on tcgen05 with T block-diagonal over the pair (the column scalings
//     folded into T, K and V rows as MN-major operands). It writes, per chunk,
//     the state kernel's shared-memory image (W, Q~ gamma, P, diag(gamma_C /
//     gamma) K, all bf16 in the canonical 128B-swizzled tile layouts, and U)
//     by bulk copies, and gamma_C to a small array beside the images.
//   gdr_state_kernel (one CTA per v-head, chunks in order): the state lives
//     transposed, S^T[v][k], in tensor memory (fp32) with a bf16 copy in shared
//     memory as the MMA operand; per chunk one bulk copy brings the chunk
//     image (prefetched two chunks ahead; it also carries U in bf16), and every contraction has M = 128
//     (v): S^T W^T (committed alone, Delta waits only for it), S^T (Q~ gamma)^T
//     (left to run under Delta), then Delta^T = U^T - S^T W^T, then O^T +=
//     Delta^T P^T and S^T = gamma_C S^T + Delta^T (diag(gamma_C/gamma) K). O^T is
//     double-buffered in TMEM; while the next chunk runs it is staged in shared
//     memory and leaves as one 3-D TMA store. One warp of the nine issues every
//     MMA and every copy, so the other eight never wait on issue.
// All MMAs are kind::f16 with both operands bf16 and fp32 accumulation.
#include "li_common.cuh"
#include "li_tc.cuh"

#include <cuda.h>
#include <cuda_bf16.h>
#include <mutex>

LI_DEFINE_TU_STATUS(prefill)

namespace li {
namespace {

constexpr int kD = 128, kC = 64;
// per-chunk image for the state kernel (bytes)
constexpr uint32_t kImgW = 0;        // W [64 t][128 k]: two [64][64] tiles
constexpr uint32_t kImgQ = 16384;    // Q~ gamma [64 t][128 k]: two tiles
constexpr uint32_t kImgP = 32768;    // P [64 i][64 j]: one tile
constexpr uint32_t kImgKd = 40960;   // (gamma_C/gamma_t) k_t as [64 t][128 k]: two MN-major tiles
constexpr uint32_t kImgU = 57344;    // U [64 t][128 v] bf16, 256-byte rows, 16-byte granules swizzled (u_off)
constexpr uint32_t kImgBytes = 73728;   // (gamma_C lives in PrefillArgs::gC)

struct PrefillArgs {
    const __nv_bfloat16 *q, *k, *v;   // [T][Hk][D], [T][Hk][D], [T][Hv][D]
    const float *g, *beta;            // [T][Hv]
    float *state;                     // [Hv][D(k)][D(v)], in/out
    float *o;                         // [T][Hv][D]
    int T, Hk, Hv, n_chunks;
    float scale;
    uint8_t *img;                     // [Hv][n_chunks][kImgBytes]
    float *gC;                        // [Hv][n_chunks] gamma_C of each chunk
};

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&v);
}
__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// byte offset of U[t][v] in the image: granule v / 8 of row t sits at granule
// (v / 8) ^ (t % 16), so row-parallel granule writes and column-parallel
// element reads are both free of bank conflicts
__host__ __device__ __forceinline__ uint32_t u_off(int t, int v) {
    return (uint32_t)(t * 256 + ((((v >> 3) ^ (t & 15))) << 4) + (v & 7) * 2);
}

// ---------------------------------------------------------------------------
// prep: one CTA per (chunk pair, v-head), 256 threads. The 128 rows of K, Q
// and V come in by TMA as [128 t][64 d] 128B-swizzled tiles (two per
// matrix); K and V serve unchanged as the MN-major B operands of W and U, and
// the column scalings diag(beta gamma), diag(beta) go into two bf16 copies of
// T. Every piece of the chunk images is finished in shared memory in its
// image layout and leaves by bulk copy.
// ---------------------------------------------------------------------------
constexpr uint32_t kPrepKt = 0, kPrepQt = 32768, kPrepVt = 65536, kPrepTk = 98304, kPrepTv = 131072,
                   kPrepPs = 163840, kPrepAf = 180224;
constexpr int kAS = 68;   // row stride of the fp32 A matrix (16-byte rows; float4 row writes are conflict-free)
constexpr uint32_t kPrepMisc = kPrepAf + 2 * 64 * kAS * 4;
constexpr size_t kPrepSmem = kPrepMisc + 8192 + 1024;

__device__ __forceinline__ void st_bf16_granules(uint8_t *tile_base, int row, int k0, const uint32_t (&r)[32]) {
    // 32 values of `row` (columns k0 .. k0+31, k0 a multiple of 32) into [rows][64] tiles by 64 columns
#pragma unroll
    for (int gg = 0; gg < 4; ++gg) {
        const int k = k0 + gg * 8;
        *reinterpret_cast<uint4 *>(tile_base + (k >> 6) * 16384 + sw128_off(row, (k & 63) >> 3)) =
            make_uint4(pack_bf16x2(__uint_as_float(r[8 * gg]), __uint_as_float(r[8 * gg + 1])),
                       pack_bf16x2(__uint_as_float(r[8 * gg + 2]), __uint_as_float(r[8 * gg + 3])),
                       pack_bf16x2(__uint_as_float(r[8 * gg + 4]), __uint_as_float(r[8 * gg + 5])),
                       pack_bf16x2(__uint_as_float(r[8 * gg + 6]), __uint_as_float(r[8 * gg + 7])));
    }
}

__device__ __forceinline__ void tma_load_3d(void *smem_dst, const CUtensorMap *map, int x, int y, int z,
                                            uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4}], [%5];"
        ::"r"(smem_addr(smem_dst)), "l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ void tma_load_2d(void *smem_dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];"
        ::"r"(smem_addr(smem_dst)), "l"(map), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ void bulk_s2g(void *gdst, const void *ssrc, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;"
                 ::"l"(gdst), "r"(smem_addr(ssrc)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void fma4(float4 &acc, float x, const float4 &y) {
    acc.x = fmaf(x, y.x, acc.x);
    acc.y = fmaf(x, y.y, acc.y);
    acc.z = fmaf(x, y.z, acc.z);
    acc.w = fmaf(x, y.w, acc.w);
}
__device__ __forceinline__ float4 ld4(const float *p) { return *reinterpret_cast<const float4 *>(p); }
__device__ __forceinline__ float f4get(const float4 &v, int e) { return e == 0 ? v.x : e == 1 ? v.y : e == 2 ? v.z : v.w; }

// acc[0..n4) += sum_{k in [k0, k1)} X[k] * Y[k][4 e ..], k0 and k1 multiples of 4;
// X a row (16-byte aligned), Y rows `ys` floats apart (16-byte aligned)
template <int N4>
__device__ __forceinline__ void row_times_rows(float4 (&acc)[N4], const float *X, const float *Y, int ys, int k0,
                                               int k1) {
#pragma unroll 1
    for (int k = k0; k < k1; k += 4) {
        const float4 x4 = ld4(X + k);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            const float xv = f4get(x4, kk);
#pragma unroll
            for (int e = 0; e < N4; ++e) fma4(acc[e], xv, ld4(Y + (k + kk) * ys + 4 * e));
        }
    }
}

// 4 consecutive columns (j0 % 4 == 0) of row i of the bf16 copies of T: T x fk -> tk, T x fv -> tv
__device__ __forceinline__ void put_t4(uint8_t *tk, uint8_t *tv, int i, int j0, float4 t, const float *fk,
                                       const float *fv) {
    const uint32_t off = sw128_off(i, j0 >> 3) + (uint32_t)(j0 & 7) * 2;
    *reinterpret_cast<uint2 *>(tk + off) =
        make_uint2(pack_bf16x2(t.x * fk[j0], t.y * fk[j0 + 1]), pack_bf16x2(t.z * fk[j0 + 2], t.w * fk[j0 + 3]));
    *reinterpret_cast<uint2 *>(tv + off) =
        make_uint2(pack_bf16x2(t.x * fv[j0], t.y * fv[j0 + 1]), pack_bf16x2(t.z * fv[j0 + 2], t.w * fv[j0 + 3]));
}

struct PrepMaps {
    CUtensorMap k, q, v;   // [T][H][128] bf16 as (d, head, token), box [128 t][64 d], 128B swizzle
    CUtensorMap g, beta;   // [T][Hv] fp32 as (head, token), box [128 t][4 heads]
    int gb_tma;            // g and beta by TMA (Hv % 4 == 0), else plain loads
};

__global__ void __launch_bounds__(256, 1) gdr_prep_kernel(PrefillArgs a, const __grid_constant__ PrepMaps maps) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *sm = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    uint8_t *Kt = sm + kPrepKt, *Qt = sm + kPrepQt, *Vt = sm + kPrepVt, *Tk = sm + kPrepTk, *Tv = sm + kPrepTv;
    uint8_t *Ps = sm + kPrepPs;                              // P image tiles of both chunks
    float *Tf = reinterpret_cast<float *>(Qt);               // [2][64][64] fp32 T, once the Q image has left
    float *Mb = reinterpret_cast<float *>(Ps), *Mc = Mb + 1024;   // block-merge temporaries, once P has left
    uint8_t *Ws = Vt, *Us = Tk;                              // W, U staging once V, T are consumed
    float *Af = reinterpret_cast<float *>(sm + kPrepAf);    // [2][64][kAS] strictly lower A
    float *gbox = reinterpret_cast<float *>(sm + kPrepMisc), *bbox = gbox + 512;   // [128 t][4 heads] g, beta (TMA)
    float *gc = bbox + 512;                                   // [128] log gamma
    float *gam = gc + 128, *bet = gam + 128, *fkd = bet + 128, *fbg = fkd + 128, *wsum = fbg + 128;   // wsum [8]
    uint64_t *bar = reinterpret_cast<uint64_t *>(wsum + 8);   // [4]: rows, K K^T + Q K^T, W + U, g + beta
    uint32_t *holder = reinterpret_cast<uint32_t *>(bar + 4);

    const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
    const int h = blockIdx.y, pair = blockIdx.x;
    const int hk = h / (a.Hv / a.Hk);
    const int t0 = pair * 2 * kC;
    const int chunk0 = 2 * pair;
    const int nc = a.n_chunks;
    const int n_valid = nc - chunk0 >= 2 ? 2 : 1;   // chunks of this pair inside the sequence
    constexpr int kStoreThread = 128;                // issues every bulk store of the CTA

    if (tid == 0) {
        for (int b = 0; b < 4; ++b) mbar_init(&bar[b], 1);
        fence_mbar_init();
        if (maps.gb_tma) {
            mbar_arrive_expect_tx(&bar[3], 2 * 2048);
            tma_load_2d(gbox, &maps.g, h & ~3, t0, &bar[3]);
            tma_load_2d(bbox, &maps.beta, h & ~3, t0, &bar[3]);
        }
        mbar_arrive_expect_tx(&bar[0], 6 * 16384);
        for (int hh = 0; hh < 2; ++hh) {
            tma_load_3d(Kt + hh * 16384, &maps.k, hh * 64, hk, t0, &bar[0]);
            tma_load_3d(Qt + hh * 16384, &maps.q, hh * 64, hk, t0, &bar[0]);
            tma_load_3d(Vt + hh * 16384, &maps.v, hh * 64, h, t0, &bar[0]);
        }
    }
    if (warp == 1) tmem_alloc(holder, 512);
    __syncthreads();   // the barriers are initialised before anyone waits on them

    // 1. decay prefix sums (per 64-token chunk), beta
    const bool gb_ok = !maps.gb_tma || mbar_wait(&bar[3], 0);
    if (tid < 128) {
        const int t = t0 + tid;
        const bool ok = t < a.T;
        float gv;
        if (maps.gb_tma) {
            gv = gbox[tid * 4 + (h & 3)];
            bet[tid] = bbox[tid * 4 + (h & 3)];
        } else {
            gv = ok ? a.g[(size_t)t * a.Hv + h] : 0.f;
            bet[tid] = ok ? a.beta[(size_t)t * a.Hv + h] : 0.f;
        }
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const float y = __shfl_up_sync(0xffffffffu, gv, o);
            if (lane >= o) gv += y;
        }
        if (lane == 31) wsum[warp] = gv;
        gc[tid] = gv;
    }
    __syncthreads();
    if (tid < 128) {
        if (warp & 1) gc[tid] += wsum[warp - 1];   // second warp of each chunk
        gam[tid] = expf(gc[tid]);
        fkd[tid] = expf(gc[(tid & 64) + 63] - gc[tid]);   // gamma_C / gamma_t
        fbg[tid] = bet[tid] * gam[tid];
    }
    // both bf16 copies of T start as zeros (only the lower blocks get written)
    for (int e = tid; e < 4096; e += 256) reinterpret_cast<uint4 *>(Tk)[e] = make_uint4(0, 0, 0, 0);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *holder;
    const uint32_t idesc = idesc_kf16(128, 128, true);
    // 2. K K^T -> cols [0,128), Q K^T -> cols [128,256)
    bool ok = mbar_wait(&bar[0], 0) && gb_ok;
    if (tid == 0 && ok) {
        tc_fence_after();
        for (int kb = 0; kb < 2; ++kb) {
            const uint64_t dk = sw128_desc(smem_addr(Kt + kb * 16384)), dq = sw128_desc(smem_addr(Qt + kb * 16384));
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                umma_f16(tmem + 0, dk + 2 * j, dk + 2 * j, idesc, (kb | j) ? 1u : 0u);
                umma_f16(tmem + 128, dq + 2 * j, dk + 2 * j, idesc, (kb | j) ? 1u : 0u);
            }
        }
        umma_commit(&bar[1]);
    }
    if (ok) ok = mbar_wait(&bar[1], 0);
    tc_fence_after();
    // 3. rows: A (fp32, shared), P (image tile), Q~ gamma (Q rows scaled in
    // place: they are the image tiles); warp w serves TMEM lane quarter w % 4
    // (row r) and column half w / 4
    const int q4 = warp & 3, half = warp >> 2;
    const int r = 32 * q4 + lane, c = r >> 6, i = r & 63;
    const uint32_t lane_addr = tmem + ((uint32_t)(32 * q4) << 16);
    if (ok) {
        uint32_t kk[32], qk[32];
        tmem_ld32_nowait(lane_addr + c * 64 + half * 32, kk);
        tmem_ld32_nowait(lane_addr + 128 + c * 64 + half * 32, qk);
        tmem_wait_ld();
        float *Arow = Af + (c * 64 + i) * kAS + half * 32;
        const float gr = gc[r], br = bet[r];
        uint32_t prow[16];
#pragma unroll
        for (int jj = 0; jj < 32; jj += 4) {
            float av[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int jl = jj + u, j = half * 32 + jl;
                const float ratio = j <= i ? expf(gr - gc[c * 64 + j]) : 0.f;
                av[u] = j < i ? br * ratio * __uint_as_float(kk[jl]) : 0.f;
                qk[jl] = __float_as_uint(a.scale * ratio * __uint_as_float(qk[jl]));
            }
            *reinterpret_cast<float4 *>(Arow + jj) = make_float4(av[0], av[1], av[2], av[3]);
            prow[jj >> 1] = pack_bf16x2(__uint_as_float(qk[jj]), __uint_as_float(qk[jj + 1]));
            prow[(jj >> 1) + 1] = pack_bf16x2(__uint_as_float(qk[jj + 2]), __uint_as_float(qk[jj + 3]));
        }
#pragma unroll
        for (int gg = 0; gg < 4; ++gg)
            *reinterpret_cast<uint4 *>(Ps + c * 8192 + sw128_off(i, half * 4 + gg)) =
                make_uint4(prow[4 * gg], prow[4 * gg + 1], prow[4 * gg + 2], prow[4 * gg + 3]);
        const float qs = a.scale * gam[r];
#pragma unroll
        for (int g8 = 0; g8 < 8; ++g8) {
            uint4 *p = reinterpret_cast<uint4 *>(Qt + half * 16384 + sw128_off(r, g8));
            const uint4 w = *p;
            *p = make_uint4(pack_bf16x2(bf16_lo(w.x) * qs, bf16_hi(w.x) * qs),
                            pack_bf16x2(bf16_lo(w.y) * qs, bf16_hi(w.y) * qs),
                            pack_bf16x2(bf16_lo(w.z) * qs, bf16_hi(w.z) * qs),
                            pack_bf16x2(bf16_lo(w.w) * qs, bf16_hi(w.w) * qs));
        }
        if (i == 63 && half == 0 && chunk0 + c < nc) a.gC[(size_t)h * nc + chunk0 + c] = gam[r];
    }
    fence_proxy_async_shared();
    if (__syncthreads_or(!ok)) ok = false;
    uint8_t *img0 = a.img + ((size_t)h * nc + chunk0) * kImgBytes;
    if (tid == kStoreThread && ok) {
        for (int cc = 0; cc < n_valid; ++cc) {
            uint8_t *img = img0 + (size_t)cc * kImgBytes;
            bulk_s2g(img + kImgP, Ps + cc * 8192, 8192);
            bulk_s2g(img + kImgQ, Qt + cc * 8192, 8192);
            bulk_s2g(img + kImgQ + 8192, Qt + 16384 + cc * 8192, 8192);
        }
        asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    }
    // 4. T = (I + A)^-1 of each chunk, by blocks: the four 16x16 diagonal
    // blocks by forward substitution (one column per thread), then the 32-wide
    // diagonal blocks T_10 = -T_11 (A_10 T_00), then the 64-wide one the same
    // way. fp32 T goes to Tf (over the Q tiles, once their image copy has been
    // read); each finished block also goes to the two bf16 copies.
    float x[16];
    if (tid < 128) {
        const int b = tid >> 4, c = b >> 2, I = b & 3, jj = tid & 15;
        const float *Ab = Af + (c * 64 + 16 * I) * kAS + 16 * I;
#pragma unroll
        for (int ii = 0; ii < 16; ++ii) x[ii] = 0.f;
#pragma unroll
        for (int ii = 0; ii < 16; ++ii) {
            float s0 = 0.f, s1 = 0.f;
#pragma unroll
            for (int kk = 0; kk < ii; kk += 4) {
                const float4 a4 = ld4(Ab + ii * kAS + kk);   // zeros from the diagonal on
                s0 = fmaf(a4.x, x[kk], s0);
                s1 = fmaf(a4.y, x[kk + 1], s1);
                s0 = fmaf(a4.z, x[kk + 2], s0);
                s1 = fmaf(a4.w, x[kk + 3], s1);
            }
            x[ii] = ii < jj ? 0.f : (ii == jj ? 1.f : -(s0 + s1));
        }
    }
    if (tid == kStoreThread) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
    __syncthreads();   // the Q and P tiles have been read: Tf and the temporaries may overwrite them
    if (ok) {
        if (tid < 128) {
            const int b = tid >> 4, c = b >> 2, I = b & 3, jj = tid & 15, j = 16 * I + jj;
            float *tcol = Tf + (c * 64 + 16 * I) * 64 + j;
            const uint32_t cb = (uint32_t)(j & 7) * 2;
            const float fk = fbg[64 * c + j], fv = bet[64 * c + j];
#pragma unroll
            for (int ii = 0; ii < 16; ++ii) {
                tcol[ii * 64] = x[ii];
                const uint32_t off = c * 16384 + sw128_off(64 * c + 16 * I + ii, j >> 3) + cb;
                *reinterpret_cast<__nv_bfloat16 *>(Tk + off) = __float2bfloat16_rn(x[ii] * fk);
                *reinterpret_cast<__nv_bfloat16 *>(Tv + off) = __float2bfloat16_rn(x[ii] * fv);
            }
        }
        __syncthreads();
        // 32-wide: block q = (chunk, pair p): I = 2p + 1, J = 2p; thread: row r, columns c0 .. c0+3
        {
            const int q = tid >> 6, c = q >> 1, I = 2 * (q & 1) + 1, J = I - 1;
            const int r = (tid >> 2) & 15, c0 = (tid & 3) * 4;
            float4 m[1] = {make_float4(0.f, 0.f, 0.f, 0.f)};
            row_times_rows<1>(m, Af + (c * 64 + 16 * I + r) * kAS + 16 * J, Tf + (c * 64 + 16 * J) * 64 + 16 * J + c0,
                              64, 0, 16);
            *reinterpret_cast<float4 *>(Mb + q * 256 + r * 16 + c0) = m[0];
            __syncthreads();
            float4 t[1] = {make_float4(0.f, 0.f, 0.f, 0.f)};
            row_times_rows<1>(t, Tf + (c * 64 + 16 * I + r) * 64 + 16 * I, Mb + q * 256 + c0, 16, 0, 16);
            t[0] = make_float4(-t[0].x, -t[0].y, -t[0].z, -t[0].w);
            *reinterpret_cast<float4 *>(Tf + (c * 64 + 16 * I + r) * 64 + 16 * J + c0) = t[0];
            put_t4(Tk + c * 16384, Tv + c * 16384, 64 * c + 16 * I + r, 16 * J + c0, t[0], fbg + 64 * c,
                   bet + 64 * c);
        }
        __syncthreads();
        // 64-wide: T_[23][01] = -T_[23][23] (A_[23][01] T_[01][01]); thread: chunk c, row r, columns c0 .. c0+7
        {
            const int c = tid >> 7, r = (tid >> 2) & 31, c0 = (tid & 3) * 8;
            float4 m[2] = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
            // T_[01][01][k][c0 ..] is zero for k < c0
            row_times_rows<2>(m, Af + (c * 64 + 32 + r) * kAS, Tf + c * 64 * 64 + c0, 64, c0, 32);
            *reinterpret_cast<float4 *>(Mc + c * 1024 + r * 32 + c0) = m[0];
            *reinterpret_cast<float4 *>(Mc + c * 1024 + r * 32 + c0 + 4) = m[1];
            __syncthreads();
            float4 t[2] = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
            // T_[23][23][r][k] is zero for k >= 16 when r < 16 (warp-uniform)
            row_times_rows<2>(t, Tf + (c * 64 + 32 + r) * 64 + 32, Mc + c * 1024 + c0, 32, 0, r < 16 ? 16 : 32);
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                t[e] = make_float4(-t[e].x, -t[e].y, -t[e].z, -t[e].w);
                put_t4(Tk + c * 16384, Tv + c * 16384, 64 * c + 32 + r, c0 + 4 * e, t[e], fbg + 64 * c, bet + 64 * c);
            }
        }
    }
    fence_proxy_async_shared();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // 5. W = (T diag(beta gamma)) K -> cols [256,384), U = (T diag(beta)) V -> cols [384,512);
    // K and V rows are the MN-major B operands (N = d in two 64-wide blocks 16 KB apart)
    if (tid == 0 && ok) {
        const uint32_t idmn = idesc | kIdescBMajorMN;
        for (int ks = 0; ks < 8; ++ks) {
            const uint64_t dtk = sw128_desc(smem_addr(Tk + (ks >> 2) * 16384)) + 2 * (ks & 3);
            const uint64_t dtv = sw128_desc(smem_addr(Tv + (ks >> 2) * 16384)) + 2 * (ks & 3);
            const uint64_t dk = sw128_mn_desc(smem_addr(Kt + ks * 2048), 16384);
            const uint64_t dv = sw128_mn_desc(smem_addr(Vt + ks * 2048), 16384);
            umma_f16(tmem + 256, dtk, dk, idmn, ks ? 1u : 0u);
            umma_f16(tmem + 384, dtv, dv, idmn, ks ? 1u : 0u);
        }
        umma_commit(&bar[2]);
    }
    if (ok) ok = mbar_wait(&bar[2], 0);
    tc_fence_after();
    // 6. W rows (warps 0-3) and U rows (warps 4-7) from TMEM to their image
    // layouts; K rows scaled by gamma_C/gamma_t in place (the K^T diag image,
    // MN-major), d-half by warp group
    if (ok) {
        const uint32_t col = half ? 384 : 256;
        for (int cb = 0; cb < 4; ++cb) {
            uint32_t w[32];
            tmem_ld32_nowait(lane_addr + col + cb * 32, w);
            tmem_wait_ld();
            if (half == 0) {
                st_bf16_granules(Ws, r, cb * 32, w);
            } else {
#pragma unroll
                for (int gg = 0; gg < 4; ++gg)
                    *reinterpret_cast<uint4 *>(Us + u_off(r, cb * 32 + gg * 8)) =
                        make_uint4(pack_bf16x2(__uint_as_float(w[8 * gg]), __uint_as_float(w[8 * gg + 1])),
                                   pack_bf16x2(__uint_as_float(w[8 * gg + 2]), __uint_as_float(w[8 * gg + 3])),
                                   pack_bf16x2(__uint_as_float(w[8 * gg + 4]), __uint_as_float(w[8 * gg + 5])),
                                   pack_bf16x2(__uint_as_float(w[8 * gg + 6]), __uint_as_float(w[8 * gg + 7])));
            }
        }
        const float kd = fkd[r];
#pragma unroll
        for (int g8 = 0; g8 < 8; ++g8) {
            uint4 *p = reinterpret_cast<uint4 *>(Kt + half * 16384 + sw128_off(r, (g8 + r) & 7));
            const uint4 w = *p;
            *p = make_uint4(pack_bf16x2(bf16_lo(w.x) * kd, bf16_hi(w.x) * kd),
                            pack_bf16x2(bf16_lo(w.y) * kd, bf16_hi(w.y) * kd),
                            pack_bf16x2(bf16_lo(w.z) * kd, bf16_hi(w.z) * kd),
                            pack_bf16x2(bf16_lo(w.w) * kd, bf16_hi(w.w) * kd));
        }
    }
    fence_proxy_async_shared();
    tc_fence_before();
    if (__syncthreads_or(!ok)) ok = false;
    if (tid == kStoreThread) {
        if (ok) {
            for (int cc = 0; cc < n_valid; ++cc) {
                uint8_t *img = img0 + (size_t)cc * kImgBytes;
                bulk_s2g(img + kImgW, Ws + cc * 8192, 8192);
                bulk_s2g(img + kImgW + 8192, Ws + 16384 + cc * 8192, 8192);
                bulk_s2g(img + kImgKd, Kt + cc * 8192, 8192);
                bulk_s2g(img + kImgKd + 8192, Kt + 16384 + cc * 8192, 8192);
                bulk_s2g(img + kImgU, Us + cc * 16384, 16384);
            }
            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        }
        asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    }
    if (!ok && tid == 0) {
        // a wait gave up: let the copies and MMAs in flight finish (bounded) before the TMEM is freed
        mbar_wait(&bar[0], 0);
        if (maps.gb_tma) mbar_wait(&bar[3], 0);
        mbar_wait(&bar[1], 0);
        mbar_wait(&bar[2], 0);
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// ---------------------------------------------------------------------------
// state: one CTA per v-head, chunks in order; 9 warps: warps 0-7 compute (warp
// w serves TMEM lane quarter w % 4, v = 32 (w % 4) + lane, and column half
// w / 4), warp 8 issues the MMAs and all TMA traffic (chunk images in, the
// chunk's outputs out as one 3-D TMA store)
// ---------------------------------------------------------------------------
constexpr uint32_t kStRing = 0, kStS = 2 * kImgBytes, kStDt = kStS + 32768, kStO = kStDt + 16384,
                   kStMisc = kStO + 32768;
constexpr size_t kStateSmem = kStMisc + 64 + 1024;

// TMA store of a [64 t][128 v] fp32 tile to o rows (t, h) (tokens past T are clipped)
__device__ __forceinline__ void tma_store_o(const CUtensorMap *m, const void *src, int h, int t0) {
    asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%1, %2, %3}], [%4];"
                 ::"l"(m), "r"(0), "r"(h), "r"(t0), "r"(smem_addr(src)) : "memory");
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

__global__ void __launch_bounds__(288, 1) gdr_state_kernel(PrefillArgs a, const __grid_constant__ CUtensorMap tmO) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *sm = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    uint8_t *ring = sm + kStRing, *St = sm + kStS, *Dt = sm + kStDt;
    float *Os = reinterpret_cast<float *>(sm + kStO);                // [64 t][128 v] output staging
    uint64_t *full = reinterpret_cast<uint64_t *>(sm + kStMisc);   // [2]
    uint64_t *mbar = full + 2;
    uint32_t *holder = reinterpret_cast<uint32_t *>(mbar + 1);

    const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
    const bool issuer = warp == 8;
    const int q4 = warp & 3, half = (warp >> 2) & 1;
    const int v = 32 * q4 + lane;
    const int h = blockIdx.x;
    const int nc = a.n_chunks;
    if (tid == 0) {
        mbar_init(&full[0], 1);
        mbar_init(&full[1], 1);
        mbar_init(mbar, 1);
        fence_mbar_init();
    }
    if (issuer) tmem_alloc(holder, 512);
    __syncthreads();
    if (issuer && lane == 0) {
        for (int n = 0; n < 2 && n < nc; ++n) {
            mbar_arrive_expect_tx(&full[n], kImgBytes);
            bulk_g2s(ring + (size_t)n * kImgBytes, a.img + ((size_t)h * nc + n) * kImgBytes, kImgBytes, &full[n]);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *holder;
    const uint32_t lane_addr = tmem + ((uint32_t)(32 * q4) << 16);
    float *Sg = a.state + (size_t)h * kD * kD;
    if (!issuer) {
        // S^T row v, columns k in this warp's half: S[k][v] -> TMEM and the bf16 operand tiles
        for (int cb = 0; cb < 2; ++cb) {
            const int k0 = half * 64 + cb * 32;
            uint32_t r[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(Sg[(size_t)(k0 + j) * kD + v]);
            tmem_st32(lane_addr + k0, r);
            st_bf16_granules(St, v, k0, r);
        }
        tmem_wait_st();
        fence_proxy_async_shared();
    }
    tc_fence_before();
    __syncthreads();

    const uint32_t id64 = idesc_kf16(128, 64, true), id128 = idesc_kf16(128, 128, true);
    // TMEM columns: S^T [0,128), S^T W^T [128,192), O^T of chunk n in [192 + 64 (n & 1), +64)
    // (double-buffered: chunk n's outputs leave while chunk n+1 runs)
    auto stage_o = [&](int m) {   // compute threads: O^T of chunk m (TMEM) -> Os[t][v]
        uint32_t o2[32];
        tmem_ld32_nowait(lane_addr + 192 + 64 * (m & 1) + half * 32, o2);
        tmem_wait_ld();
#pragma unroll
        for (int t = 0; t < 32; ++t) Os[(half * 32 + t) * kD + v] = __uint_as_float(o2[t]);
    };
    float gC_next = (!issuer && nc > 0) ? a.gC[(size_t)h * nc] : 1.f;
    uint32_t mph = 0;
    int n = 0;
    for (; n < nc; ++n) {
        const int b = n & 1;
        const uint8_t *img = ring + (size_t)b * kImgBytes;
        const uint32_t d2col = 192 + 64 * (uint32_t)b;
        const float gC = gC_next;
        if (!issuer && n + 1 < nc) gC_next = a.gC[(size_t)h * nc + n + 1];
        bool ok = mbar_wait(&full[b], (uint32_t)((n >> 1) & 1));
        if (issuer && lane == 0) {
            asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");   // the last output store has left Os
        }
        if (__syncthreads_or(!ok)) break;
        tc_fence_after();
        if (issuer) {
            if (lane == 0) {
                // S^T W^T -> cols [128,192), committed alone (Delta needs only it);
                // then S^T (Q~ gamma)^T -> this chunk's O^T buffer
                for (int kb = 0; kb < 2; ++kb) {
                    const uint64_t ds = sw128_desc(smem_addr(St + kb * 16384));
                    const uint64_t dw = sw128_desc(smem_addr(img + kImgW + kb * 8192));
#pragma unroll
                    for (int j = 0; j < 4; ++j) umma_f16(tmem + 128, ds + 2 * j, dw + 2 * j, id64, (kb | j) ? 1u : 0u);
                }
                umma_commit(mbar);
                for (int kb = 0; kb < 2; ++kb) {
                    const uint64_t ds = sw128_desc(smem_addr(St + kb * 16384));
                    const uint64_t dq = sw128_desc(smem_addr(img + kImgQ + kb * 8192));
#pragma unroll
                    for (int j = 0; j < 4; ++j) umma_f16(tmem + d2col, ds + 2 * j, dq + 2 * j, id64, (kb | j) ? 1u : 0u);
                }
            }
        } else {
            // the previous chunk's outputs to the staging tile, U^T (this thread's 32
            // tokens), S^T *= gamma_C (its 64 columns), then Delta^T = U^T - S^T W^T
            if (n > 0) stage_o(n - 1);
            float u[32];
            {
#pragma unroll
                for (int t = 0; t < 32; ++t)
                    u[t] = __bfloat162float(*reinterpret_cast<const __nv_bfloat16 *>(img + kImgU + u_off(half * 32 + t, v)));
            }
            for (int cb = 0; cb < 2; ++cb) {
                const uint32_t col = half * 64 + cb * 32;
                uint32_t r[32];
                tmem_ld32_nowait(lane_addr + col, r);
                tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(__uint_as_float(r[j]) * gC);
                tmem_st32(lane_addr + col, r);
            }
            tmem_wait_st();
            ok = mbar_wait(mbar, mph);
            tc_fence_after();
            uint32_t d1[32];
            tmem_ld32_nowait(lane_addr + 128 + half * 32, d1);
            tmem_wait_ld();
#pragma unroll
            for (int t = 0; t < 32; ++t) d1[t] = __float_as_uint(u[t] - __uint_as_float(d1[t]));
#pragma unroll
            for (int gg = 0; gg < 4; ++gg)
                *reinterpret_cast<uint4 *>(Dt + sw128_off(v, half * 4 + gg)) =
                    make_uint4(pack_bf16x2(__uint_as_float(d1[8 * gg]), __uint_as_float(d1[8 * gg + 1])),
                               pack_bf16x2(__uint_as_float(d1[8 * gg + 2]), __uint_as_float(d1[8 * gg + 3])),
                               pack_bf16x2(__uint_as_float(d1[8 * gg + 4]), __uint_as_float(d1[8 * gg + 5])),
                               pack_bf16x2(__uint_as_float(d1[8 * gg + 6]), __uint_as_float(d1[8 * gg + 7])));
            fence_proxy_async_shared();   // Dt and Os writes -> the MMAs' and the TMA store's reads
        }
        mph ^= 1;
        tc_fence_before();
        if (__syncthreads_or(!ok)) break;
        tc_fence_after();
        if (issuer && lane == 0) {
            // O^T += Delta^T P^T; S^T += Delta^T (diag(gamma_C/gamma) K); one commit covers
            // every MMA of the chunk (the image slot and Delta are free when it arrives)
            const uint64_t dd = sw128_desc(smem_addr(Dt));
            const uint64_t dp = sw128_desc(smem_addr(img + kImgP));
#pragma unroll
            for (int j = 0; j < 4; ++j) umma_f16(tmem + d2col, dd + 2 * j, dp + 2 * j, id64, 1u);
            // B = diag(gamma_C/gamma) K rows, MN-major (two 64-wide k blocks 8 KB apart)
#pragma unroll
            for (int j = 0; j < 4; ++j)
                umma_f16(tmem + 0, dd + 2 * j, sw128_mn_desc(smem_addr(img + kImgKd + j * 2048), 8192),
                         id128 | kIdescBMajorMN, 1u);
            umma_commit(mbar);
            if (n > 0) tma_store_o(&tmO, Os, h, (n - 1) * kC);   // the previous chunk's outputs
        }
        if (!issuer) {
            ok = mbar_wait(mbar, mph);
            tc_fence_after();
            // the next chunk's bf16 S^T operand
            for (int cb = 0; cb < 2; ++cb) {
                const int k0 = half * 64 + cb * 32;
                uint32_t r[32];
                tmem_ld32_nowait(lane_addr + k0, r);
                tmem_wait_ld();
                st_bf16_granules(St, v, k0, r);
            }
            fence_proxy_async_shared();
        }
        mph ^= 1;
        tc_fence_before();
        if (__syncthreads_or(!ok)) break;
        // ring slot b is free (every MMA reading it has completed): chunk n+2 goes there
        if (issuer && lane == 0 && n + 2 < nc) {
            mbar_arrive_expect_tx(&full[b], kImgBytes);
            bulk_g2s(ring + (size_t)b * kImgBytes, a.img + ((size_t)h * nc + n + 2) * kImgBytes, kImgBytes, &full[b]);
        }
    }
    tc_fence_after();
    const bool done = n == nc;
    if (done) {
        if (issuer && lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
        __syncthreads();
        if (!issuer) {
            stage_o(nc - 1);
            fence_proxy_async_shared();
            // final state S[k][v] from S^T in TMEM
            for (int cb = 0; cb < 2; ++cb) {
                const int k0 = half * 64 + cb * 32;
                uint32_t r[32];
                tmem_ld32_nowait(lane_addr + k0, r);
                tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 32; ++j) Sg[(size_t)(k0 + j) * kD + v] = __uint_as_float(r[j]);
            }
        }
        __syncthreads();
        if (issuer && lane == 0) tma_store_o(&tmO, Os, h, (nc - 1) * kC);
    } else if (issuer && lane == 0) {
        // a wait gave up: let the copies and MMAs in flight finish (bounded) before exit
        for (int m = n; m < n + 2 && m < nc; ++m) mbar_wait(&full[m & 1], (uint32_t)((m >> 1) & 1));
        mbar_wait(mbar, mph);
    }
    if (issuer && lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");   // outputs written
    tc_fence_before();
    __syncthreads();
    if (issuer) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
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

// [T][H][128] rows as a 3-D tensor (d, head, token) with a [tokens][1][128 or 64 d] box
int encode_rows(CUtensorMap *m, void *base, bool bf16, int T, int H, int box_d, int box_t) {
    EncodeTiledFn fn = encoder();
    if (!fn) return LI_ERR_UNSUPPORTED;
    const cuuint64_t es = bf16 ? 2 : 4;
    const cuuint64_t dims[3] = {(cuuint64_t)kD, (cuuint64_t)H, (cuuint64_t)T};
    const cuuint64_t strides[2] = {(cuuint64_t)kD * es, (cuuint64_t)H * kD * es};
    const cuuint32_t box[3] = {(cuuint32_t)box_d, 1, (cuuint32_t)box_t};
    const cuuint32_t estr[3] = {1, 1, 1};
    const CUresult r = fn(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, base, dims,
                          strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          bf16 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                          bf16 ? CU_TENSOR_MAP_L2_PROMOTION_L2_256B : CU_TENSOR_MAP_L2_PROMOTION_NONE,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : LI_ERR_BAD_SHAPE;
}

// [T][Hv] fp32 per-head scalars as a 2-D tensor (head, token), box [2 chunks of tokens][4 heads]
int encode_heads(CUtensorMap *m, float *base, int T, int Hv) {
    EncodeTiledFn fn = encoder();
    if (!fn) return LI_ERR_UNSUPPORTED;
    const cuuint64_t dims[2] = {(cuuint64_t)Hv, (cuuint64_t)T};
    const cuuint64_t strides[1] = {(cuuint64_t)Hv * 4};
    const cuuint32_t box[2] = {4, (cuuint32_t)(2 * kC)};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, base, dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : LI_ERR_BAD_SHAPE;
}

template <typename K>
int set_smem(K kern, size_t bytes) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    return (int)e;
}

}  // namespace
}  // namespace li

using namespace li;

extern "C" {

size_t li_deltanet_chunk_prefill_workspace_size(int T, int n_v_heads, int head_dim) {
    if (T <= 0 || n_v_heads <= 0 || head_dim != kD) return 0;
    const size_t nc = (size_t)(T + kC - 1) / kC;
    return (size_t)n_v_heads * nc * kImgBytes + ((size_t)n_v_heads * nc * 4 + 255) / 256 * 256;
}

int li_launch_deltanet_chunk_prefill_bf16(const void *q, const void *k, const void *v, const float *g,
                                          const float *beta, float *state, float *o, int T, int n_k_heads,
                                          int n_v_heads, int head_dim, float scale, void *workspace,
                                          size_t workspace_bytes, void *stream) {
    if (!q || !k || !v || !g || !beta || !state || !o || T < 0 || n_k_heads <= 0 || n_v_heads <= 0)
        return LI_ERR_BAD_ARG;
    if (head_dim != kD) return LI_ERR_UNSUPPORTED;
    if (n_v_heads % n_k_heads) return LI_ERR_BAD_SHAPE;
    if (T == 0) return 0;
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(workspace)) return LI_ERR_MISALIGNED;
    if (!workspace || workspace_bytes < li_deltanet_chunk_prefill_workspace_size(T, n_v_heads, head_dim))
        return LI_ERR_WORKSPACE;
    static std::once_flag once;
    static int attr_rc = 0;
    std::call_once(once, [] {
        attr_rc = set_smem(gdr_prep_kernel, kPrepSmem);
        if (!attr_rc) attr_rc = set_smem(gdr_state_kernel, kStateSmem);
    });
    if (attr_rc) return attr_rc;
    int rc0 = 0;
    PrefillArgs a = {};
    a.q = (const __nv_bfloat16 *)q; a.k = (const __nv_bfloat16 *)k; a.v = (const __nv_bfloat16 *)v;
    a.g = g; a.beta = beta; a.state = state; a.o = o;
    a.T = T; a.Hk = n_k_heads; a.Hv = n_v_heads; a.n_chunks = (T + kC - 1) / kC; a.scale = scale;
    a.img = (uint8_t *)workspace;
    a.gC = (float *)((uint8_t *)workspace + (size_t)n_v_heads * a.n_chunks * kImgBytes);
    if (!aligned16(o)) return LI_ERR_MISALIGNED;
    CUtensorMap tmO;
    PrepMaps maps;
    if ((rc0 = encode_rows(&tmO, o, false, T, n_v_heads, kD, kC)) ||
        (rc0 = encode_rows(&maps.k, const_cast<void *>(k), true, T, n_k_heads, 64, 2 * kC)) ||
        (rc0 = encode_rows(&maps.q, const_cast<void *>(q), true, T, n_k_heads, 64, 2 * kC)) ||
        (rc0 = encode_rows(&maps.v, const_cast<void *>(v), true, T, n_v_heads, 64, 2 * kC)))
        return rc0;
    maps.gb_tma = n_v_heads % 4 == 0 && aligned16(g) && aligned16(beta);
    if (maps.gb_tma &&
        ((rc0 = encode_heads(&maps.g, const_cast<float *>(g), T, n_v_heads)) ||
         (rc0 = encode_heads(&maps.beta, const_cast<float *>(beta), T, n_v_heads))))
        return rc0;
    const cudaStream_t s = (cudaStream_t)stream;
    gdr_prep_kernel<<<dim3((unsigned)((a.n_chunks + 1) / 2), (unsigned)n_v_heads), 256, kPrepSmem, s>>>(a, maps);
    int rc = launch_status();
    if (rc) return rc;
    gdr_state_kernel<<<(unsigned)n_v_heads, 288, kStateSmem, s>>>(a, tmO);
    return launch_status();
}

}  // extern "C"
