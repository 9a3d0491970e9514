// Batched-decode projections on the 5th-generation tensor cores (tcgen05).
//
// Y[b][n] = sum_k X[b][k] * W[n][k] for B >= kTcMinRows batch rows, W raw
// ggml Q4_K / Q8_0 rows. Swap-AB: the weight rows are the MMA's M side (128
// per CTA tile), the batch is N (padded to a multiple of 32, up to 256).
//
// One CTA per 128-row weight tile, 10 warps:
//   warp 4G producer: 2-D tiled TMA of raw weight blocks ([128 rows] x one
//           256-value column: 144 B Q4_K / 272 B Q8_0 per row) and of the f16
//           X tile (64 k x N rows, 128-byte swizzle) into shared-memory rings;
//   warps 0..4G-1 dequant: raw blocks -> f16 weights written in the canonical
//           K-major 128B-swizzled UMMA layout (one 16-byte granule per store,
//           bank-conflict free); group g (4 warps, one row each per
//           thread) takes k-blocks g, g+G, ... into A slot g (G = 2 or 4);
//   warp 4G+1 MMA: allocates TMEM, issues tcgen05.mma kind::f16 (fp32
//           accumulators in TMEM, N columns per weight matrix), commits slot
//           releases to mbarriers;
//   warps 0..4G-1 epilogue: tcgen05.ld 32x32b of their TMEM lane quarter, scale by
//           the X row scale, store / SwiGLU / DeltaNet conv epilogue.
// Dequant: nibbles / bytes become f16 through the 0x6400 magic-exponent form
// (one byte permute + one LOP3 per pair), then (q - 1024) * d*sc - dmin*m in
// packed half2 arithmetic (Q8_0: (u - 1152) * d). The values are rounded to
// f16 once, the products and sums are exact/fp32 in the tensor core.
//
// Weights are requested before griddepcontrol.wait (they do not depend on
// the previous kernel) and dequantized right away; X and all global writes
// come after it. Every mbarrier wait is bounded; on a timeout the CTA raises
// the device flag, skips the remaining work, drains its copies and frees its
// TMEM before returning.
#include "li_common.cuh"
#include "li_tcgemm.cuh"

#include <cuda.h>   // CUtensorMap and its enums; the encoder is fetched at run time

#include <cstring>
#include <mutex>

LI_DEFINE_TU_STATUS(tcgemm)

namespace li {
namespace {

constexpr int kBM = 128;                 // weight rows per tile
// Dequant groups of 4 warps (one tile row per thread). The group count G
// equals the number of A slots (2 or 4): group g owns slot g and its
// k-blocks g, g+G, ..., so each slot's successive phases are produced and
// awaited by one group and no parity wait can run two phases ahead.
constexpr int kMaxGroups = 4;
constexpr int kMaxThreads = (4 * kMaxGroups + 2) * kWarp;
constexpr int kMaxSmem = 227 * 1024;

struct TcPlan {
    int NW;          // weight matrices per tile (2: SwiGLU gate/up)
    int RB;          // raw bytes per row per raw stage (one 256-value column)
    int Npad;        // batch columns
    int RS, AS, XS;  // ring depths
    int tiles;       // CTAs
    int seg_tiles[3];
    int tmem_cols;
    int n_raw;       // raw stages (K / 256)
    int ks;          // K splits (CTAs per tile); > 1 only for kTcStore, reduced with fp32 red.add
    int raw_per_split;
    uint32_t off_a, off_x, off_raw, off_bar;
    size_t smem;
};

// ---------------------------------------------------------------------------
// PTX wrappers
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(void *smem_dst, const CUtensorMap *map, int x, int y,
                                            uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];"
        ::"r"(smem_addr(smem_dst)), "l"(map), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t *holder, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(smem_addr(holder)), "r"(ncols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16, cta_group::1.
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
        ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u),
          "r"(0u)
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
          "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (SBO), version 1 (sm_100).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor: fp32 accumulate, f16 A and B, both K-major, M=128.
__host__ __device__ constexpr uint32_t idesc_f16(int n) {
    return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
}

// Byte offset of 16-byte granule g (0..7) of row m in a 128B-swizzled
// K-major tile (8-row atoms of 1024 bytes).
__device__ __forceinline__ uint32_t sw128_off(int m, int g) {
    return (uint32_t)((m >> 3) * 1024 + (m & 7) * 128 + ((g ^ (m & 7)) << 4));
}

__device__ __forceinline__ uint32_t lop3_or_and(uint32_t a, uint32_t mask, uint32_t orv) {
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(mask), "r"(orv));   // (a & b) | c
    return r;
}

__device__ __forceinline__ __half2 h2_bits(uint32_t v) { return *reinterpret_cast<__half2 *>(&v); }
__device__ __forceinline__ uint32_t bits_h2(__half2 v) { return *reinterpret_cast<uint32_t *>(&v); }

// Q4_K: row m's 64 weights of sub-block pair `sub` of the staged super-block
// (header at +0, nibbles at +16 + 32*sub) -> 8 granules of the A tile.
__device__ __forceinline__ void dequant_q4k_row(const uint8_t *raw_row, int sub, uint8_t *a_tile, int m) {
    const uint4 h = *reinterpret_cast<const uint4 *>(raw_row);
    const uint4 q0 = *reinterpret_cast<const uint4 *>(raw_row + 16 + 32 * sub);
    const uint4 q1 = *reinterpret_cast<const uint4 *>(raw_row + 32 + 32 * sub);
    const uint32_t bsh = 16u * (uint32_t)(sub & 1);
    const uint32_t a0 = h.y >> bsh, a1 = h.z >> bsh, a2 = h.w >> bsh;
    uint32_t sc0, sc1, m0, m1;
    if (sub < 2) {
        sc0 = a0 & 63u; sc1 = (a0 >> 8) & 63u; m0 = a1 & 63u; m1 = (a1 >> 8) & 63u;
    } else {
        sc0 = (a2 & 15u) | ((a0 >> 2) & 48u);
        sc1 = ((a2 >> 8) & 15u) | ((a0 >> 10) & 48u);
        m0 = ((a2 >> 4) & 15u) | ((a1 >> 2) & 48u);
        m1 = ((a2 >> 12) & 15u) | ((a1 >> 10) & 48u);
    }
    const float d = half_bits_to_float(h.x), dmin = half_bits_to_float(h.x >> 16);
    // low nibbles: (1024+q) - 1024; high nibbles sit 4 bits up: (1024+16q) - 1024, scale/16
    const __half2 dl0 = __float2half2_rn(d * (float)sc0);
    const __half2 ml0 = __float2half2_rn(-dmin * (float)m0);
    const __half2 dl1 = __float2half2_rn(d * (float)sc1 * 0.0625f);
    const __half2 ml1 = __float2half2_rn(-dmin * (float)m1);
    const __half2 magic = h2_bits(0x64006400u);
    const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
    for (int g = 0; g < 4; ++g) {
        uint32_t lo[4], hi[4];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const uint32_t x = w[2 * g + j];
            const uint32_t t01 = __byte_perm(x, 0u, 0x4140u);   // bytes 0,1 -> halves
            const uint32_t t23 = __byte_perm(x, 0u, 0x4342u);   // bytes 2,3 -> halves
            lo[2 * j] = bits_h2(__hfma2(__hsub2(h2_bits(lop3_or_and(t01, 0x000F000Fu, 0x64006400u)), magic), dl0, ml0));
            lo[2 * j + 1] = bits_h2(__hfma2(__hsub2(h2_bits(lop3_or_and(t23, 0x000F000Fu, 0x64006400u)), magic), dl0, ml0));
            hi[2 * j] = bits_h2(__hfma2(__hsub2(h2_bits(lop3_or_and(t01, 0x00F000F0u, 0x64006400u)), magic), dl1, ml1));
            hi[2 * j + 1] = bits_h2(__hfma2(__hsub2(h2_bits(lop3_or_and(t23, 0x00F000F0u, 0x64006400u)), magic), dl1, ml1));
        }
        *reinterpret_cast<uint4 *>(a_tile + sw128_off(m, g)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        *reinterpret_cast<uint4 *>(a_tile + sw128_off(m, 4 + g)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    }
}

// Q8_0: row m's blocks 2*sub and 2*sub+1 of the staged 8-block column
// (row copy 16-byte aligned, blocks 34 bytes apart) -> 8 granules.
__device__ __forceinline__ void dequant_q80_row(const uint8_t *raw_row, int sub, uint8_t *a_tile, int m) {
#pragma unroll
    for (int bb = 0; bb < 2; ++bb) {
        const uint32_t off = 34u * (uint32_t)(2 * sub + bb);
        const uint32_t *wp = reinterpret_cast<const uint32_t *>(raw_row + (off & ~3u));
        uint32_t v[9];
#pragma unroll
        for (int i = 0; i < 9; ++i) v[i] = wp[i];
        const bool odd = (off & 2u) != 0;
        const uint32_t sh = odd ? 32u : 16u;
        const uint32_t dbits = odd ? (v[0] >> 16) : (v[0] & 0xffffu);
        const __half2 d2 = h2_bits(dbits | (dbits << 16));
        const __half2 bias = h2_bits(0x64806480u);          // 1152 = 1024 + 128
#pragma unroll
        for (int g = 0; g < 4; ++g) {
            uint32_t o[4];
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const uint32_t q = __funnelshift_rc(v[2 * g + j], v[2 * g + j + 1], sh) ^ 0x80808080u;
                const uint32_t p01 = __byte_perm(q, 0x00006464u, 0x5140u);
                const uint32_t p23 = __byte_perm(q, 0x00006464u, 0x5342u);
                o[2 * j] = bits_h2(__hmul2(__hsub2(h2_bits(p01), bias), d2));
                o[2 * j + 1] = bits_h2(__hmul2(__hsub2(h2_bits(p23), bias), d2));
            }
            *reinterpret_cast<uint4 *>(a_tile + sw128_off(m, 4 * bb + g)) = make_uint4(o[0], o[1], o[2], o[3]);
        }
    }
}

// Bounded wait that gives up at once when the CTA has already aborted.
__device__ __forceinline__ bool wait_or_abort(uint64_t *bar, uint32_t parity, volatile int *abort_flag) {
    if (*abort_flag) return false;
    if (!mbar_wait(bar, parity)) {
        *abort_flag = 1;
        return false;
    }
    return true;
}

template <int WT, int EPI>
__global__ void __launch_bounds__(kMaxThreads, 1)
tc_gemm_kernel(const __grid_constant__ CUtensorMap tmW0, const __grid_constant__ CUtensorMap tmW1,
               const __grid_constant__ CUtensorMap tmW2, const __grid_constant__ CUtensorMap tmX,
               TcArgs a, TcPlan p) {
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte aligned base for the swizzled tiles
    uint8_t *smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    constexpr int NW = EPI == kTcSwiGLU ? 2 : 1;
    const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
    const int G = p.AS;                                   // dequant groups = A slots
    const int deq_warps = 4 * G, producer_warp = deq_warps, mma_warp = deq_warps + 1;

    uint8_t *a_ring = smem + p.off_a;      // [AS][NW][16 KB]
    uint8_t *x_ring = smem + p.off_x;      // [XS][Npad*128]
    uint8_t *raw_ring = smem + p.off_raw;  // [RS][NW][128*RB]
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + p.off_bar);
    uint64_t *raw_full = bars, *raw_empty = raw_full + p.RS;
    uint64_t *a_full = raw_empty + p.RS, *a_empty = a_full + p.AS;
    uint64_t *x_full = a_empty + p.AS, *x_empty = x_full + p.XS;
    uint64_t *acc_full = x_empty + p.XS;
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(acc_full + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);

    // CTA -> (segment, first row, K split)
    const int split = (int)blockIdx.x % p.ks;
    int tile = (int)blockIdx.x / p.ks, seg = 0;
    if (a.n_seg > 1 && tile >= p.seg_tiles[0]) {
        tile -= p.seg_tiles[0];
        seg = 1;
        if (a.n_seg > 2 && tile >= p.seg_tiles[1]) { tile -= p.seg_tiles[1]; seg = 2; }
    }
    const int row0 = tile * kBM;
    const int seg_rows = seg == 0 ? a.seg_rows[0] : (seg == 1 ? a.seg_rows[1] : a.seg_rows[2]);
    float *const dseg = seg == 0 ? a.dst[0] : (seg == 1 ? a.dst[1] : a.dst[2]);
    const int dstride = seg == 0 ? a.dst_stride[0] : (seg == 1 ? a.dst_stride[1] : a.dst_stride[2]);
    const CUtensorMap *tmA = seg == 0 ? &tmW0 : (seg == 1 ? &tmW1 : &tmW2);
    const CUtensorMap *tmB = &tmW1;                       // SwiGLU: up matrix
    const int r_base = split * p.raw_per_split;           // first raw stage (256 k) of this CTA
    const int n_raw = p.raw_per_split;
    const int nkb = n_raw * 4;                            // 64-value k-blocks
    const uint32_t raw_stage_bytes = (uint32_t)(kBM * p.RB);
    const uint32_t x_slot_bytes = (uint32_t)(p.Npad * 128);

    if (threadIdx.x == 0) {
        for (int i = 0; i < p.RS; ++i) { mbar_init(&raw_full[i], 1); mbar_init(&raw_empty[i], deq_warps); }   // every dequant warp once per raw stage
        for (int i = 0; i < p.AS; ++i) { mbar_init(&a_full[i], kBM); mbar_init(&a_empty[i], 1); }
        for (int i = 0; i < p.XS; ++i) { mbar_init(&x_full[i], 1); mbar_init(&x_empty[i], 1); }
        mbar_init(acc_full, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == mma_warp) tmem_alloc(tmem_holder, (uint32_t)p.tmem_cols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;
    grid_dep_launch_dependents();

    if (warp == producer_warp) {
        if (lane == 0) {
            int issued_raw = 0, issued_x = 0;
            auto issue_raw = [&](int r) {
                const int s = r % p.RS;
                if (r >= p.RS && !wait_or_abort(&raw_empty[s], (uint32_t)(((r / p.RS) - 1) & 1), abort_flag))
                    return false;
                mbar_arrive_expect_tx(&raw_full[s], (uint32_t)NW * raw_stage_bytes);
                uint8_t *dst = raw_ring + (size_t)s * NW * raw_stage_bytes;
                tma_load_2d(dst, tmA, (r_base + r) * (p.RB / 2), row0, &raw_full[s]);
                if (NW == 2) tma_load_2d(dst + raw_stage_bytes, tmB, (r_base + r) * (p.RB / 2), row0, &raw_full[s]);
                issued_raw = r + 1;
                return true;
            };
            // weights do not depend on the previous kernel: prefetch them first
            const int pre = p.RS < n_raw ? p.RS : n_raw;
            for (int r = 0; r < pre; ++r) issue_raw(r);
            grid_dep_wait();
            for (int kb = 0; kb < nkb && !*abort_flag; ++kb) {
                const int s = kb % p.XS;
                if (kb >= p.XS && !wait_or_abort(&x_empty[s], (uint32_t)(((kb / p.XS) - 1) & 1), abort_flag))
                    break;
                mbar_arrive_expect_tx(&x_full[s], x_slot_bytes);
                tma_load_2d(x_ring + (size_t)s * x_slot_bytes, &tmX, (r_base * 4 + kb) * 64, 0, &x_full[s]);
                issued_x = kb + 1;
                // keep the raw ring RS stages ahead of the X stream
                const int want = kb / 4 + p.RS;
                while (issued_raw < n_raw && issued_raw < want && !*abort_flag) issue_raw(issued_raw);
            }
            // drain: every copy this CTA issued has landed before it exits
            for (int r = issued_raw - p.RS < 0 ? 0 : issued_raw - p.RS; r < issued_raw; ++r)
                mbar_wait(&raw_full[r % p.RS], (uint32_t)((r / p.RS) & 1));
            for (int kb = issued_x - p.XS < 0 ? 0 : issued_x - p.XS; kb < issued_x; ++kb)
                mbar_wait(&x_full[kb % p.XS], (uint32_t)((kb / p.XS) & 1));
        }
    } else if (warp == mma_warp) {
        if (lane == 0) {
            const uint32_t idesc = idesc_f16(p.Npad);
            for (int kb = 0; kb < nkb; ++kb) {
                const int as = kb % p.AS, xs = kb % p.XS;
                if (!wait_or_abort(&a_full[as], (uint32_t)((kb / p.AS) & 1), abort_flag)) break;
                if (!wait_or_abort(&x_full[xs], (uint32_t)((kb / p.XS) & 1), abort_flag)) break;
                tc_fence_after();
                const uint64_t bdesc = sw128_desc(smem_addr(x_ring + (size_t)xs * x_slot_bytes));
#pragma unroll
                for (int w = 0; w < NW; ++w) {
                    const uint64_t adesc = sw128_desc(smem_addr(a_ring + ((size_t)as * NW + w) * 16384));
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        umma_f16(tmem + (uint32_t)(w * p.Npad), adesc + 2 * j, bdesc + 2 * j, idesc,
                                 (kb > 0 || j > 0) ? 1u : 0u);
                }
                umma_commit(&a_empty[as]);
                umma_commit(&x_empty[xs]);
            }
            umma_commit(acc_full);   // also orders every MMA issued before TMEM is read or freed
        }
    } else {
        // ---------------- dequant warps ----------------
        const int grp = warp / 4;                 // k-blocks grp, grp+G, ...
        const int m = threadIdx.x % kBM;          // tile row
        for (int kb = grp; kb < nkb; kb += G) {
            const int r = kb / 4, sub = kb % 4;
            const int rs = r % p.RS, as = kb % p.AS;
            if (!wait_or_abort(&raw_full[rs], (uint32_t)((r / p.RS) & 1), abort_flag)) break;
            if (kb >= p.AS && !wait_or_abort(&a_empty[as], (uint32_t)(((kb / p.AS) - 1) & 1), abort_flag))
                break;
            const uint8_t *raw = raw_ring + (size_t)rs * NW * raw_stage_bytes;
#pragma unroll
            for (int w = 0; w < NW; ++w) {
                const uint8_t *row = raw + (size_t)w * raw_stage_bytes + (size_t)m * p.RB;
                uint8_t *at = a_ring + ((size_t)as * NW + w) * 16384;
                if (WT == LI_WTYPE_Q4_K) dequant_q4k_row(row, sub, at, m);
                else dequant_q80_row(row, sub, at, m);
            }
            fence_proxy_async_shared();           // generic-proxy writes -> tensor core reads
            mbar_arrive(&a_full[as]);
            if (sub + G >= 4) {                   // the group's last k-block of this raw stage
                __syncwarp();
                if (lane == 0) mbar_arrive(&raw_empty[rs]);
            }
        }

        // ---------------- epilogue ----------------
        grid_dep_wait();                          // outputs may be read by the previous kernel
        const bool ok = wait_or_abort(acc_full, 0u, abort_flag);
        tc_fence_after();
        const int q = warp & 3, part = warp >> 2;
        const int rloc = 32 * q + lane;           // tile row of this thread's TMEM lane
        const int row = row0 + rloc;
        const bool row_ok = ok && row < seg_rows;
        float4 cw = make_float4(0.f, 0.f, 0.f, 0.f);
        if (EPI == kTcConv && row_ok && row < a.conv_channels)
            cw = *reinterpret_cast<const float4 *>(a.conv_w + 4 * (size_t)row);
        const int cols = p.Npad / G;              // batch columns of this warp
        const bool conv_row = EPI == kTcConv && row_ok && row < a.conv_channels;
        for (int c0 = part * cols; c0 < (part + 1) * cols; c0 += 8) {
            uint32_t acc[8], acc2[8];
            const uint32_t taddr = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)c0;
            if (ok) {
                tmem_ld8(taddr, acc);
                if (NW == 2) tmem_ld8(taddr + (uint32_t)p.Npad, acc2);
            }
            if (!row_ok) continue;
            // every load of the chunk is issued before the first use
            float sc[8], cst[8][3];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int b = c0 + i;
                sc[i] = (a.xscale && b < a.B) ? a.xscale[b] : 1.0f;
                if (conv_row && b < a.B) {
                    const float *cs = a.conv_state + ((size_t)b * a.conv_channels + row) * 3;
                    cst[i][0] = cs[0]; cst[i][1] = cs[1]; cst[i][2] = cs[2];
                }
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int b = c0 + i;
                if (b >= a.B) continue;
                const float v = __uint_as_float(acc[i]) * sc[i];
                if (EPI == kTcSwiGLU) {
                    const float u = __uint_as_float(acc2[i]) * sc[i];
                    a.dst[0][(size_t)b * a.dst_stride[0] + row] = silu(v) * u;
                } else if (EPI == kTcStore) {
                    float *d = dseg + (size_t)b * dstride + row;
                    if (p.ks > 1) atomicAdd(d, v); else *d = v;
                } else {
                    float out = v;
                    if (conv_row) {
                        float *cs = a.conv_state + ((size_t)b * a.conv_channels + row) * 3;
                        const float accv = fmaf(cw.x, cst[i][0], fmaf(cw.y, cst[i][1], fmaf(cw.z, cst[i][2], cw.w * v)));
                        cs[0] = cst[i][1];
                        cs[1] = cst[i][2];
                        cs[2] = v;
                        out = silu(accv);
                    }
                    a.dst[0][(size_t)b * a.dst_stride[0] + row] = out;
                }
            }
        }
    }

    if (*abort_flag && threadIdx.x == 0) atomicExch(&g_device_error, LI_ERR_TIMEOUT);
    tc_fence_before();
    __syncthreads();
    if (warp == mma_warp) {
        // an aborted CTA may not have waited for its MMAs: wait (bounded) before freeing TMEM
        if (*abort_flag && lane == 0) mbar_wait(acc_full, 0u);
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, (uint32_t)p.tmem_cols);
    }
}

// ---------------------------------------------------------------------------
// x -> f16 with optional RMSNorm and a per-row power-of-two scale
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256)
tc_prep_kernel(const float *__restrict__ x, int x_stride, const float *__restrict__ gamma, float eps, int K,
               __half *__restrict__ X16, float *__restrict__ xscale) {
    __shared__ float s_sq[8], s_mx[8];
    const int b = blockIdx.x, t = threadIdx.x;
    grid_dep_wait();
    const float4 *x4 = reinterpret_cast<const float4 *>(x + (size_t)b * x_stride);
    const float4 *g4 = reinterpret_cast<const float4 *>(gamma);
    float sq = 0.f, mx = 0.f;
    for (int i = t; i < K / 4; i += 256) {
        const float4 v = x4[i];
        sq = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, sq))));
        float4 g = gamma ? g4[i] : make_float4(1.f, 1.f, 1.f, 1.f);
        mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x * g.x), fabsf(v.y * g.y)), fmaxf(fabsf(v.z * g.z), fabsf(v.w * g.w))));
    }
    sq = warp_sum(sq);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((t & 31) == 0) { s_sq[t >> 5] = sq; s_mx[t >> 5] = mx; }
    __syncthreads();
    float tot = 0.f, m = 0.f;
    for (int i = 0; i < 8; ++i) { tot += s_sq[i]; m = fmaxf(m, s_mx[i]); }
    const float r = gamma ? rsqrtf(tot / (float)K + eps) : 1.0f;
    m *= r;
    // s = 2^e with max/s in [2^13, 2^14): inside f16 range with room to spare
    int e = 0;
    if (m > 0.f) { frexpf(m, &e); e -= 14; }
    const float s = ldexpf(1.0f, e), inv = ldexpf(1.0f, -e) * r;
    if (t == 0) xscale[b] = s;
    __half2 *o2 = reinterpret_cast<__half2 *>(X16 + (size_t)b * K);
    for (int i = t; i < K / 4; i += 256) {
        const float4 v = x4[i];
        const float4 g = gamma ? g4[i] : make_float4(1.f, 1.f, 1.f, 1.f);
        o2[2 * i] = __floats2half2_rn(v.x * g.x * inv, v.y * g.y * inv);
        o2[2 * i + 1] = __floats2half2_rn(v.z * g.z * inv, v.w * g.w * inv);
    }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
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

int encode_2d(CUtensorMap *map, CUtensorMapDataType dt, const void *base, uint64_t inner, uint64_t rows,
              uint64_t row_bytes, uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle sw) {
    EncodeTiledFn fn = encoder();
    if (!fn) return LI_ERR_UNSUPPORTED;
    const cuuint64_t dims[2] = {inner, rows};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {box_inner, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(map, dt, 2, const_cast<void *>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : LI_ERR_BAD_SHAPE;
}

int plan(const TcArgs &a, TcPlan *p) {
    if (a.wtype != LI_WTYPE_Q4_K && a.wtype != LI_WTYPE_Q8_0) return LI_ERR_UNSUPPORTED;
    if (a.K <= 0 || a.K % 256 || a.B <= 0 || a.B > 256) return LI_ERR_BAD_SHAPE;
    p->NW = a.epi == kTcSwiGLU ? 2 : 1;
    p->RB = a.wtype == LI_WTYPE_Q4_K ? 144 : 272;
    p->Npad = (a.B + 31) / 32 * 32;
    p->n_raw = a.K / 256;
    int cols = 32;
    while (cols < p->NW * p->Npad) cols <<= 1;
    if (cols > 512) return LI_ERR_BAD_SHAPE;
    p->tmem_cols = cols;
    p->tiles = 0;
    for (int s = 0; s < 3; ++s) {
        p->seg_tiles[s] = s < a.n_seg ? (a.seg_rows[s] + kBM - 1) / kBM : 0;
        p->tiles += p->seg_tiles[s];
    }
    // K splits: fill the SMs when there are few tiles (plain stores only;
    // the partial sums meet in fp32 reductions into a zeroed output)
    p->ks = 1;
    if (a.epi == kTcStore) {
        int sms = 148;
        int dev = 0;
        if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        while (p->ks * 2 * p->tiles <= sms && p->n_raw % (p->ks * 2) == 0 && p->n_raw / (p->ks * 2) >= 2)
            p->ks *= 2;
    }
    p->raw_per_split = p->n_raw / p->ks;
    // rings: raw 3 (2 for two weight matrices), A 4, X as deep as fits (<= 16 k-blocks)
    const size_t raw_b = (size_t)p->NW * kBM * p->RB, a_b = (size_t)p->NW * 16384, x_b = (size_t)p->Npad * 128;
    const size_t fixed = 1024 + 512;   // alignment slack, barriers, TMEM holder
    for (int rs = p->NW == 2 ? 2 : 3; rs >= 2; --rs) {
        for (int as = 4; as >= 2; as -= 2) {   // slot kb % AS; each phase is filled by one group
            const size_t used = rs * raw_b + as * a_b + fixed;
            if (used + 2 * x_b > (size_t)kMaxSmem) continue;
            int xs = (int)(((size_t)kMaxSmem - used) / x_b);
            if (xs > 16) xs = 16;
            p->RS = rs; p->AS = as; p->XS = xs;
            p->off_a = 0;
            p->off_x = (uint32_t)(as * a_b);
            p->off_raw = p->off_x + (uint32_t)(xs * x_b);
            p->off_bar = p->off_raw + (uint32_t)(rs * raw_b);
            p->smem = p->off_bar + 8 * (2 * rs + 2 * as + 2 * xs + 1) + 16 + 1024;
            if (p->smem <= (size_t)kMaxSmem) return 0;
        }
    }
    return LI_ERR_BAD_SHAPE;
}

template <int WT, int EPI>
int launch_kernel(const CUtensorMap *maps, const TcArgs &a, const TcPlan &p, cudaStream_t stream, bool pdl) {
    auto kern = tc_gemm_kernel<WT, EPI>;
    static std::once_flag once;
    static cudaError_t attr_err = cudaSuccess;
    std::call_once(once, [&] {
        attr_err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem);
    });
    if (attr_err != cudaSuccess) return (int)attr_err;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(p.tiles * p.ks));
    cfg.blockDim = dim3((unsigned)((4 * p.AS + 2) * kWarp));
    cfg.dynamicSmemBytes = p.smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return (int)cudaLaunchKernelEx(&cfg, kern, maps[0], maps[1], maps[2], maps[3], a, p);
}

}  // namespace

int tc_prep_launch(const float *x, int x_stride, const float *gamma, float eps, int B, int K, __half *X16,
                   float *xscale, cudaStream_t stream, bool pdl) {
    if (K % 8 || !aligned16(x) || (gamma && !aligned16(gamma)) || !aligned16(X16)) return LI_ERR_MISALIGNED;
    return (int)launch_pdl(tc_prep_kernel, dim3((unsigned)B), dim3(256), 0, stream, pdl, x, x_stride, gamma, eps,
                           K, X16, xscale);
}

bool tc_gemm_splits_k(const TcArgs &a) {
    TcPlan p;
    return plan(a, &p) == 0 && p.ks > 1;
}

int tc_gemm_launch(const TcArgs &a, cudaStream_t stream, bool pdl) {
    TcPlan p;
    int rc = plan(a, &p);
    if (rc) return rc;
    const size_t rb = li_row_bytes(a.wtype, a.K);
    CUtensorMap maps[4];
    memset(maps, 0, sizeof(maps));
    const int nw = a.epi == kTcSwiGLU ? 2 : a.n_seg;
    for (int s = 0; s < 3; ++s) {
        const int src = s < nw ? s : 0;
        const int rows = a.epi == kTcSwiGLU ? a.seg_rows[0] : a.seg_rows[src];
        if (!aligned16(a.W[src])) return LI_ERR_MISALIGNED;
        rc = encode_2d(&maps[s], CU_TENSOR_MAP_DATA_TYPE_UINT16, a.W[src], rb / 2, (uint64_t)rows, rb,
                       (uint32_t)(p.RB / 2), kBM, CU_TENSOR_MAP_SWIZZLE_NONE);
        if (rc) return rc;
    }
    if (!aligned16(a.X16)) return LI_ERR_MISALIGNED;
    rc = encode_2d(&maps[3], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a.X16, (uint64_t)a.K, (uint64_t)a.B,
                   (uint64_t)a.K * 2, 64, (uint32_t)p.Npad, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    const bool q4 = a.wtype == LI_WTYPE_Q4_K;
    switch (a.epi) {
    case kTcStore: return q4 ? launch_kernel<LI_WTYPE_Q4_K, kTcStore>(maps, a, p, stream, pdl)
                              : launch_kernel<LI_WTYPE_Q8_0, kTcStore>(maps, a, p, stream, pdl);
    case kTcSwiGLU: return q4 ? launch_kernel<LI_WTYPE_Q4_K, kTcSwiGLU>(maps, a, p, stream, pdl)
                               : launch_kernel<LI_WTYPE_Q8_0, kTcSwiGLU>(maps, a, p, stream, pdl);
    case kTcConv: return q4 ? launch_kernel<LI_WTYPE_Q4_K, kTcConv>(maps, a, p, stream, pdl)
                             : launch_kernel<LI_WTYPE_Q8_0, kTcConv>(maps, a, p, stream, pdl);
    default: return LI_ERR_BAD_ARG;
    }
}

}  // namespace li
