// Batched-decode projections on the 5th-generation tensor cores (tcgen05).
//
// Y[b][n] = sum_k X[b][k] * W[n][k] for B >= kTcMinRows batch rows, W raw
// ggml Q4_K / Q8_0 rows. Swap-AB: the weight rows are the MMA's M side (128
// per CTA tile), the batch is N (padded to a multiple of 32, up to 256).
//
// One CTA per 128-row weight tile (and K split), (WPG+1)G+2 warps in G groups
// of WPG = 4 or 8 dequant warps:
//   warps WPG*g .. WPG*g+WPG-1 (group g) dequant: take k-blocks g, g+G, ...
//           (per tile) and write them as f16 into the group's A slots, one
//           tile row per thread (WPG 8: two warps per lane quarter, 32 k
//           each): into tensor memory (tcgen05.st, the row's 64 k in 32
//           columns of its TMEM lane) when the TMEM has room next to the
//           accumulators, else into shared memory (canonical K-major
//           128B-swizzled UMMA layout, one 16-byte granule per store,
//           bank-conflict free);
//   warp WPG*G+g (group g) MMA issuer, lane 0: issues tcgen05.mma kind::f16
//           into the group's own fp32 accumulators in TMEM, commits slot
//           releases, and releases raw stages and X slots once per group.
//   warp (WPG+1)G producer of the weights: allocates TMEM; lane 0 streams
//           2-D tiled TMA boxes of raw weight blocks ([128 rows] x SB
//           256-value columns: 144 B Q4_K / 272 B Q8_0 per row and column)
//           into a ring of raw stages;
//   warp (WPG+1)G+1 producer of X: lane 0 bulk-copies slots of f16 X
//           k-blocks (64 k x N rows each, 128-byte swizzle: X arrives tiled,
//           see tiled_x_offset) into a ring of X slots. Two warps, so that a
//           blocking wait of one stream never holds up the other.
//   The groups share only the raw and X rings. Epilogue (dequant warps): tcgen05.ld
//   32x32b of their TMEM lane quarter, the G partial sums added in group
//   order, scaled by the X row scale, then store / SwiGLU / DeltaNet conv.
// SwiGLU runs either with both weight matrices in every tile (each group
// dequantizes and multiplies the gate and the up rows, two accumulators per
// group) or, where the tensor memory holds twice the groups that way, as a
// pair of tiles per CTA: tile 0 the gate rows, tile 1 the same rows of the up
// matrix, each X k-block feeding both, and the epilogue multiplying
// silu(gate) by up across the two tiles' accumulators.
// Dequant: nibbles / bytes become f16 through the 0x6400 magic-exponent form
// (one byte permute + one LOP3 per pair), then (q - 1024) * d*sc - dmin*m in
// packed half2 arithmetic (Q8_0: (u - 1152) * d). The values are rounded to
// f16 once, the products and sums are exact/fp32 in the tensor core.
//
// Weights are requested before griddepcontrol.wait (they do not depend on
// the previous kernel) and dequantized right away; X and all global writes
// come after it. Every mbarrier wait is bounded; on a timeout the CTA raises
// the device flag, skips the remaining work, drains its copies and frees its
// TMEM after its MMAs have finished.
#include "li_common.cuh"
#include "li_tc.cuh"
#include "li_tcgemm.cuh"

#include <cuda.h>   // CUtensorMap and its enums; the encoder is fetched at run time

#include <cstring>
#include <mutex>

LI_DEFINE_TU_STATUS(tcgemm)

namespace li {
namespace {

constexpr int kBM = 128;                 // weight rows per tile
// Dequant + MMA groups of 4 warps (one tile row per thread). Each group owns
// its A slots and X slots, so every barrier's successive phases are awaited
// in order by one owner and no parity wait can run two phases ahead.
constexpr int kMaxGroups = 4;
constexpr int kMaxThreads = (5 * kMaxGroups + 2) * kWarp;
// Tiles per CTA the planner may choose. The kernel takes two (every X k-block
// then feeds both, with K split over three CTAs per tile pair so 147 CTAs
// cover the SMs), but measured on B200 at 64 sequences, hidden 4096, the
// DeltaNet layer step got slower: 108.8 us against 87.3 (in-projection 23.9
// us + its conv pass 6.6 us against 26.4 us in one kernel; out-projection 14.2
// against 11.6 us with twice the fp32 reductions).
constexpr int kMaxTilesPerCta = 1;
constexpr int kMaxSmem = 227 * 1024;
// Internal epilogue id: SwiGLU with the gate and up matrices as the two tiles
// of a CTA (one weight matrix per tile, one accumulator per group).
constexpr int kTcSwiGLUPair = 3;

struct TcPlan {
    int NW;          // weight matrices per tile (2: SwiGLU gate/up)
    int SB;          // 256-value columns (super-blocks) per raw stage
    int CB;          // bytes of one column per row (144 Q4_K, 272 Q8_0)
    int RB;          // raw bytes per row per raw stage (SB * CB)
    int Npad;        // batch columns
    int G;           // dequant + MMA groups (WPG dequant warps each), G = T * H
    int WPG;         // dequant warps per group: 4, or 8 (each thread then takes 32 k of a k-block)
    int T, H;        // 128-row tiles per CTA; k-phases per tile (group g: tile g / H, k-blocks g % H + H*i)
    int RS, AG;      // raw stages, A slots per group
    int XM, XS;      // X slots of H*XM k-blocks (XM per group), XS of them
    int atm;         // 1: A slots in tensor memory (32 columns each), else in shared memory
    int pair;        // 1: SwiGLU as a gate tile + an up tile per CTA (T = 2, NW = 1)
    int tiles;       // 128-row tiles over all segments (pair: gate and up tiles)
    int seg_tiles[3];
    int tmem_cols;
    int n_raw;       // raw stages over the whole K (K / (256 * SB))
    int ks;          // K splits (CTAs per tile group), the stages split as evenly as they go; > 1 only
                     // for kTcStore and kTcConv: partial sums meet by fp32 red.add in a zeroed
                     // output (kTcConv: the conv epilogue then runs in tc_conv_finish_kernel)
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

// Instruction descriptor: fp32 accumulate, f16 A and B, both K-major, M=128.
__host__ __device__ constexpr uint32_t idesc_f16(int n) { return idesc_kf16(kBM, n, false); }

__device__ __forceinline__ uint32_t lop3_or_and(uint32_t a, uint32_t mask, uint32_t orv) {
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(mask), "r"(orv));   // (a & b) | c
    return r;
}

__device__ __forceinline__ __half2 h2_bits(uint32_t v) { return *reinterpret_cast<__half2 *>(&v); }
__device__ __forceinline__ uint32_t bits_h2(__half2 v) { return *reinterpret_cast<uint32_t *>(&v); }

// Q4_K: row m's 64 weights of sub-block pair `sub` of the staged super-block
// (header at +0, nibbles at +16 + 32*sub) -> o[4*gi + t], granule gi = 0..7
// of the row's 128-byte A line (k 8*gi .. 8*gi+7).
__device__ __forceinline__ void dequant_q4k_regs(const uint8_t *raw_row, int sub, uint32_t (&o)[32]) {
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
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const uint32_t x = w[2 * g + j];
            const uint32_t t01 = __byte_perm(x, 0u, 0x4140u);   // bytes 0,1 -> halves
            const uint32_t t23 = __byte_perm(x, 0u, 0x4342u);   // bytes 2,3 -> halves
            o[4 * g + 2 * j] = bits_h2(__hfma2(__hsub2(h2_bits(lop3_or_and(t01, 0x000F000Fu, 0x64006400u)), magic), dl0, ml0));
            o[4 * g + 2 * j + 1] = bits_h2(__hfma2(__hsub2(h2_bits(lop3_or_and(t23, 0x000F000Fu, 0x64006400u)), magic), dl0, ml0));
            o[16 + 4 * g + 2 * j] = bits_h2(__hfma2(__hsub2(h2_bits(lop3_or_and(t01, 0x00F000F0u, 0x64006400u)), magic), dl1, ml1));
            o[16 + 4 * g + 2 * j + 1] = bits_h2(__hfma2(__hsub2(h2_bits(lop3_or_and(t23, 0x00F000F0u, 0x64006400u)), magic), dl1, ml1));
        }
    }
}

// Q8_0: row m's blocks 2*sub and 2*sub+1 of the staged 8-block column
// (row copy 16-byte aligned, blocks 34 bytes apart) -> o[4*gi + t].
__device__ __forceinline__ void dequant_q80_regs(const uint8_t *raw_row, int sub, uint32_t (&o)[32]) {
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
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const uint32_t q = __funnelshift_rc(v[2 * g + j], v[2 * g + j + 1], sh) ^ 0x80808080u;
                const uint32_t p01 = __byte_perm(q, 0x00006464u, 0x5140u);
                const uint32_t p23 = __byte_perm(q, 0x00006464u, 0x5342u);
                o[16 * bb + 4 * g + 2 * j] = bits_h2(__hmul2(__hsub2(h2_bits(p01), bias), d2));
                o[16 * bb + 4 * g + 2 * j + 1] = bits_h2(__hmul2(__hsub2(h2_bits(p23), bias), d2));
            }
        }
    }
}

template <int WT>
__device__ __forceinline__ void dequant_regs(const uint8_t *raw_row, int sub, uint32_t (&o)[32]) {
    if (WT == LI_WTYPE_Q4_K) dequant_q4k_regs(raw_row, sub, o);
    else dequant_q80_regs(raw_row, sub, o);
}

// Half of a 64-value k-block: k 32*hf .. 32*hf+31 of row m (Q4_K: the low
// nibbles of the pair's 32 bytes for hf = 0, the high ones for hf = 1; Q8_0:
// block 2*sub+hf) -> o[4*gi + t], granule gi = 0..3 of that half.
__device__ __forceinline__ void dequant_q4k_half(const uint8_t *raw_row, int sub, int hf, uint32_t (&o)[16]) {
    const uint4 h = *reinterpret_cast<const uint4 *>(raw_row);
    const uint4 q0 = *reinterpret_cast<const uint4 *>(raw_row + 16 + 32 * sub);
    const uint4 q1 = *reinterpret_cast<const uint4 *>(raw_row + 32 + 32 * sub);
    const uint32_t bsh = 16u * (uint32_t)(sub & 1);
    const uint32_t a0 = h.y >> bsh, a1 = h.z >> bsh, a2 = h.w >> bsh;
    uint32_t sc, mn;
    if (sub < 2) {
        sc = hf ? (a0 >> 8) & 63u : a0 & 63u;
        mn = hf ? (a1 >> 8) & 63u : a1 & 63u;
    } else {
        sc = hf ? ((a2 >> 8) & 15u) | ((a0 >> 10) & 48u) : (a2 & 15u) | ((a0 >> 2) & 48u);
        mn = hf ? ((a2 >> 12) & 15u) | ((a1 >> 10) & 48u) : ((a2 >> 4) & 15u) | ((a1 >> 2) & 48u);
    }
    const float d = half_bits_to_float(h.x), dmin = half_bits_to_float(h.x >> 16);
    // low nibbles: (1024+q) - 1024; high nibbles sit 4 bits up: (1024+16q) - 1024, scale/16
    const __half2 dl = __float2half2_rn(hf ? d * (float)sc * 0.0625f : d * (float)sc);
    const __half2 ml = __float2half2_rn(-dmin * (float)mn);
    const __half2 magic = h2_bits(0x64006400u);
    const uint32_t mask = hf ? 0x00F000F0u : 0x000F000Fu;
    const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
    for (int g = 0; g < 4; ++g) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const uint32_t x = w[2 * g + j];
            const uint32_t t01 = __byte_perm(x, 0u, 0x4140u);   // bytes 0,1 -> halves
            const uint32_t t23 = __byte_perm(x, 0u, 0x4342u);   // bytes 2,3 -> halves
            o[4 * g + 2 * j] = bits_h2(__hfma2(__hsub2(h2_bits(lop3_or_and(t01, mask, 0x64006400u)), magic), dl, ml));
            o[4 * g + 2 * j + 1] = bits_h2(__hfma2(__hsub2(h2_bits(lop3_or_and(t23, mask, 0x64006400u)), magic), dl, ml));
        }
    }
}

__device__ __forceinline__ void dequant_q80_half(const uint8_t *raw_row, int sub, int hf, uint32_t (&o)[16]) {
    const uint32_t off = 34u * (uint32_t)(2 * sub + hf);
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
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const uint32_t q = __funnelshift_rc(v[2 * g + j], v[2 * g + j + 1], sh) ^ 0x80808080u;
            const uint32_t p01 = __byte_perm(q, 0x00006464u, 0x5140u);
            const uint32_t p23 = __byte_perm(q, 0x00006464u, 0x5342u);
            o[4 * g + 2 * j] = bits_h2(__hmul2(__hsub2(h2_bits(p01), bias), d2));
            o[4 * g + 2 * j + 1] = bits_h2(__hmul2(__hsub2(h2_bits(p23), bias), d2));
        }
    }
}

template <int WT>
__device__ __forceinline__ void dequant_half(const uint8_t *raw_row, int sub, int hf, uint32_t (&o)[16]) {
    if (WT == LI_WTYPE_Q4_K) dequant_q4k_half(raw_row, sub, hf, o);
    else dequant_q80_half(raw_row, sub, hf, o);
}

// Warp-wide store of 16 registers per lane into 16 consecutive TMEM columns
// of the warp's lane quarter.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
        ::"r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
          "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}

// The 8 granules of row m into the 128B-swizzled A tile (bank-conflict free:
// the 8 rows of an atom put granule gi in 8 different 16-byte bank groups).
__device__ __forceinline__ void store_row(uint8_t *a_tile, int m, const uint32_t (&o)[32]) {
#pragma unroll
    for (int gi = 0; gi < 8; ++gi)
        *reinterpret_cast<uint4 *>(a_tile + sw128_off(m, gi)) =
            make_uint4(o[4 * gi], o[4 * gi + 1], o[4 * gi + 2], o[4 * gi + 3]);
}

// Granules 4*hf .. 4*hf+3 of row m (one half of its 64 k) into the A tile.
__device__ __forceinline__ void store_half_row(uint8_t *a_tile, int m, int hf, const uint32_t (&o)[16]) {
#pragma unroll
    for (int gi = 0; gi < 4; ++gi)
        *reinterpret_cast<uint4 *>(a_tile + sw128_off(m, 4 * hf + gi)) =
            make_uint4(o[4 * gi], o[4 * gi + 1], o[4 * gi + 2], o[4 * gi + 3]);
}

// Bounded wait that gives up at once when the CTA has already aborted.
__device__ __forceinline__ bool wait_or_abort(uint64_t *bar, uint32_t parity, volatile int *abort_flag) {
    if (mbar_try_wait(bar, parity)) return true;   // a completed phase needs no abort check
    if (*abort_flag) return false;
    if (!mbar_wait(bar, parity)) {
        *abort_flag = 1;
        return false;
    }
    return true;
}

// The same wait taken by a whole warp, with one verdict for all its lanes (the
// warp-collective steps after it need every lane on the same path).
__device__ __forceinline__ bool warp_wait_or_abort(uint64_t *bar, uint32_t parity, volatile int *abort_flag) {
    return __all_sync(0xffffffffu, wait_or_abort(bar, parity, abort_flag));
}

template <int WT, int EPI, bool ATM, int WPG>
__global__ void __launch_bounds__(kMaxThreads, 1)
tc_gemm_kernel(const __grid_constant__ CUtensorMap tmW0, const __grid_constant__ CUtensorMap tmW1,
               const __grid_constant__ CUtensorMap tmW2, TcArgs a, TcPlan p) {
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte aligned base for the swizzled tiles
    uint8_t *smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    constexpr int NW = EPI == kTcSwiGLU ? 2 : 1;
    constexpr bool PAIR = EPI == kTcSwiGLUPair;         // tile 0: gate rows, tile 1: the same up rows
    const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
    const int G = p.G, T = p.T, H = p.H;                 // groups = T tiles x H k-phases
    // WPG dequant warps per group: 4 (a thread dequantizes its row's 64 k of
    // a k-block) or 8 (32 k each, the two halves in two warps of the same
    // lane quarter); the issuers and the producer follow them
    const int issuer0 = WPG * G, producer_warp = (WPG + 1) * G, x_warp = producer_warp + 1;

    uint8_t *a_ring = smem + p.off_a;      // [G*AG][NW][16 KB] (A in shared memory)
    uint8_t *x_ring = smem + p.off_x;      // [XS][H*XM][Npad*128]
    uint8_t *raw_ring = smem + p.off_raw;  // [RS][NW][T][128*RB]
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + p.off_bar);
    uint64_t *raw_full = bars, *raw_empty = raw_full + p.RS;
    uint64_t *a_full = raw_empty + p.RS, *a_empty = a_full + G * p.AG;
    uint64_t *x_full = a_empty + G * p.AG, *x_empty = x_full + p.XS;
    uint64_t *acc_full = x_empty + p.XS;
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(acc_full + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);

    // CTA -> (segment, first of its T tiles, K split); T > 1 only with one segment
    const int split = (int)blockIdx.x % p.ks;
    int tile = (int)blockIdx.x / p.ks * T, seg = 0;
    if (a.n_seg > 1 && tile >= p.seg_tiles[0]) {
        tile -= p.seg_tiles[0];
        seg = 1;
        if (a.n_seg > 2 && tile >= p.seg_tiles[1]) { tile -= p.seg_tiles[1]; seg = 2; }
    }
    // first row of the CTA's first tile (pair: of both tiles)
    const int row0 = PAIR ? (int)blockIdx.x / p.ks * kBM : tile * kBM;
    const int seg_rows = seg == 0 ? a.seg_rows[0] : (seg == 1 ? a.seg_rows[1] : a.seg_rows[2]);
    float *const dseg = seg == 0 ? a.dst[0] : (seg == 1 ? a.dst[1] : a.dst[2]);
    const int dstride = seg == 0 ? a.dst_stride[0] : (seg == 1 ? a.dst_stride[1] : a.dst_stride[2]);
    const CUtensorMap *tmA = seg == 0 ? &tmW0 : (seg == 1 ? &tmW1 : &tmW2);
    const CUtensorMap *tmB = &tmW1;                       // SwiGLU: up matrix
    // this CTA's raw stages (256*SB k each): split s takes [s*n/ks, (s+1)*n/ks)
    const int r_base = (int)((long long)split * p.n_raw / p.ks);
    const int n_raw = (int)((long long)(split + 1) * p.n_raw / p.ks) - r_base;
    const int kpr = 4 * p.SB;                             // k-blocks per raw stage (a multiple of H)
    const int nkb = n_raw * kpr;                          // 64-value k-blocks of this CTA
    const uint32_t raw_tile_bytes = (uint32_t)(kBM * p.RB);          // one tile of one matrix
    const uint32_t raw_stage_bytes = (uint32_t)(NW * T) * raw_tile_bytes;
    const uint32_t xkb_bytes = (uint32_t)(p.Npad * 128);  // one X k-block
    const int XK = H * p.XM;                              // k-blocks per X slot (divides kpr)
    const uint32_t x_slot_bytes = (uint32_t)XK * xkb_bytes;
    const uint32_t acc_cols = (uint32_t)(NW * p.Npad);   // TMEM columns of one group's accumulators
    // A in tensor memory: slot (group, a, w) = 32 columns after all accumulators
    const uint32_t a_col0 = (uint32_t)G * acc_cols;

    if (threadIdx.x == 0) {
        for (int i = 0; i < p.RS; ++i) { mbar_init(&raw_full[i], 1); mbar_init(&raw_empty[i], G); }
        for (int i = 0; i < G * p.AG; ++i) { mbar_init(&a_full[i], WPG); mbar_init(&a_empty[i], 1); }
        for (int i = 0; i < p.XS; ++i) { mbar_init(&x_full[i], 1); mbar_init(&x_empty[i], G); }
        mbar_init(acc_full, G);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == producer_warp) tmem_alloc(tmem_holder, (uint32_t)p.tmem_cols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;
    grid_dep_launch_dependents();

    // Ring positions advance incrementally (no divisions in the loops): a
    // ring slot's fill parity flips each time its ring wraps; each A slot
    // keeps its own parity bit.
    // The weight stages and the X slots come from two warps (lane 0 each): a
    // blocking wait of one stream (griddepcontrol.wait, a ring slot) must not
    // hold the other back, as divergent lanes of one warp would.
    if (warp == producer_warp) {
        if (lane == 0) {
            // weight stages: they do not depend on the previous kernel, so no
            // griddepcontrol.wait here
            int issued = 0, s = 0;
            uint32_t par = 0;
            for (int r = 0; r < n_raw; ++r) {
                if (r >= p.RS && !wait_or_abort(&raw_empty[s], par ^ 1u, abort_flag)) break;
                mbar_arrive_expect_tx(&raw_full[s], raw_stage_bytes);
                uint8_t *dst = raw_ring + (size_t)s * raw_stage_bytes;
                // rows past the matrix (a last tile of a pair) come in as zeros
                for (int t = 0; t < T; ++t)
                    tma_load_2d(dst + (size_t)t * raw_tile_bytes, PAIR ? (t == 0 ? &tmW0 : &tmW1) : tmA,
                                (r_base + r) * (p.RB / 4), PAIR ? row0 : row0 + t * kBM, &raw_full[s]);
                if (NW == 2) tma_load_2d(dst + raw_tile_bytes, tmB, (r_base + r) * (p.RB / 4), row0, &raw_full[s]);
                issued = r + 1;
                if (++s == p.RS) { s = 0; par ^= 1u; }
                if (r + 1 == (p.RS < n_raw ? p.RS : n_raw) && EPI == kTcConv && p.ks == 1 &&
                    row0 < a.conv_channels && a.conv_channels % 4 == 0 && ((uintptr_t)a.conv_state & 15u) == 0) {
                    // once the ring is full: the epilogue's conv-state rows
                    // into L2 while the tile runs. They were last written by
                    // the previous step (finished before this step's first,
                    // non-dependent launch) and come from DRAM otherwise. A
                    // bulk prefetch needs 16-byte aligned rows of a multiple
                    // of 16 bytes: 4k channels of 12 bytes.
                    const int nrow = a.conv_channels - row0 < T * kBM ? a.conv_channels - row0 : T * kBM;
                    for (int b = 0; b < a.B; ++b)
                        bulk_prefetch_l2(a.conv_state + ((size_t)b * a.conv_channels + row0) * 3,
                                         (uint32_t)nrow * 12u);
                }
            }
            // drain: every copy issued has landed before the CTA exits
            for (int r = issued - p.RS < 0 ? 0 : issued - p.RS; r < issued; ++r)
                mbar_wait(&raw_full[r % p.RS], (uint32_t)((r / p.RS) & 1));
        }
    } else if (warp == x_warp) {
        if (lane == 0) {
            // X slots of XK consecutive k-blocks: the tiled X keeps them
            // contiguous, one bulk copy each; slot j is free again when every
            // group has committed its MMAs on it
            grid_dep_wait();                      // X is written by the previous kernel
            const uint8_t *xg = reinterpret_cast<const uint8_t *>(a.X16) + (size_t)r_base * kpr * xkb_bytes;
            const int n_xs = nkb / XK;
            int issued = 0, s = 0;
            uint32_t par = 0;
            for (int j = 0; j < n_xs; ++j) {
                if (j >= p.XS && !wait_or_abort(&x_empty[s], par ^ 1u, abort_flag)) break;
                mbar_arrive_expect_tx(&x_full[s], x_slot_bytes);
                bulk_g2s(x_ring + (size_t)s * x_slot_bytes, xg + (size_t)j * x_slot_bytes, x_slot_bytes, &x_full[s]);
                issued = j + 1;
                if (++s == p.XS) { s = 0; par ^= 1u; }
            }
            for (int j = issued - p.XS < 0 ? 0 : issued - p.XS; j < issued; ++j)
                mbar_wait(&x_full[j % p.XS], (uint32_t)((j / p.XS) & 1));
        }
    } else if (warp >= issuer0) {
        // ------------- MMA issuer of group grp (lane 0) -------------
        // Issues the group's MMAs (k-blocks grp, grp+G, ...) into its own
        // accumulators (TMEM columns [grp*acc_cols, (grp+1)*acc_cols)),
        // releases A slots, X slots (after its last k-block in the slot) and
        // raw stages (after its dequant warps are past them). The MMA issue
        // is serial in this thread, so descriptors advance by constants.
        const int grp = warp - issuer0, hph = grp % H;
        if (lane == 0) {
            const int n_it = nkb / H;
            const uint32_t idesc = idesc_f16(p.Npad);
            const uint32_t d_tmem = tmem + (uint32_t)grp * acc_cols;
            const uint64_t xdesc0 = sw128_desc(smem_addr(x_ring));
            const uint32_t xstep = xkb_bytes >> 4;     // descriptor units per X k-block
            int ai = 0, xm = 0, xs = 0, kx = hph, kin = hph, rst = 0;
            uint32_t apar = 0, xpar = 0;
            for (int i = 0; i < n_it; ++i) {
                const int slot = grp * p.AG + ai;
                if (!wait_or_abort(&a_full[slot], (apar >> ai) & 1u, abort_flag)) break;
                apar ^= 1u << ai;
                // the dequant warps have read this group's last k-block of the raw stage
                if (kin + H >= kpr) mbar_arrive(&raw_empty[rst]);
                if (xm == 0 && !wait_or_abort(&x_full[xs], xpar, abort_flag)) break;
                tc_fence_after();
                const uint64_t bdesc = xdesc0 + (uint64_t)((xs * XK + kx) * xstep);
                const uint32_t acc0 = i > 0 ? 1u : 0u;
#pragma unroll
                for (int w = 0; w < NW; ++w) {
                    if constexpr (ATM) {
                        const uint32_t at = tmem + a_col0 + (uint32_t)((slot * NW + w) * 32);
#pragma unroll
                        for (int j = 0; j < 4; ++j)
                            umma_f16_ta(d_tmem + (uint32_t)(w * p.Npad), at + (uint32_t)(8 * j), bdesc + 2 * j, idesc,
                                        j > 0 ? 1u : acc0);
                    } else {
                        const uint64_t adesc =
                            sw128_desc(smem_addr(a_ring + ((size_t)slot * NW + w) * 16384));
#pragma unroll
                        for (int j = 0; j < 4; ++j)
                            umma_f16(d_tmem + (uint32_t)(w * p.Npad), adesc + 2 * j, bdesc + 2 * j, idesc,
                                     j > 0 ? 1u : acc0);
                    }
                }
                umma_commit(&a_empty[slot]);
                if (xm == p.XM - 1) umma_commit(&x_empty[xs]);
                ai = ai + 1 == p.AG ? 0 : ai + 1;
                if (++xm == p.XM) {
                    xm = 0;
                    if (++xs == p.XS) { xs = 0; xpar ^= 1u; }
                }
                kx += H;
                if (kx >= XK) kx -= XK;
                kin += H;
                if (kin >= kpr) {
                    kin -= kpr;
                    if (++rst == p.RS) rst = 0;
                }
            }
            // every MMA this group issued has finished when acc_full sees this commit
            umma_commit(acc_full);
        }
    } else {
        // ---------------- dequant warps ----------------
        // Group grp (4 warps, one tile row per thread) dequantizes k-blocks
        // grp, grp+G, ... into its A slots; the values are computed before
        // the slot is known free, so the wait overlaps the arithmetic.
        const int grp = warp / WPG, tdx = grp / H;
        const int hf = (warp % WPG) >> 2;         // WPG 8: which 32 k of each k-block
        const int m = threadIdx.x % kBM;          // row of tile tdx
        int ai = 0, kin = grp % H, rst = 0;
        uint32_t epar = 0, rpar = 0;
        bool new_stage = true;
        for (int i = 0; i < nkb / H; ++i) {
            const int slot = grp * p.AG + ai;
            if (new_stage) {
                if (!warp_wait_or_abort(&raw_full[rst], rpar, abort_flag)) break;
                new_stage = false;
            }
            // super-block column kin/4, sub-block pair (Q8_0: blocks) kin%4
            const uint8_t *row = raw_ring + (size_t)rst * raw_stage_bytes + (size_t)tdx * raw_tile_bytes +
                                 (size_t)m * p.RB + (size_t)(kin >> 2) * p.CB;
            if constexpr (WPG == 8) {
                uint32_t o[16];
                dequant_half<WT>(row, kin & 3, hf, o);
                if (i >= p.AG) {
                    if (!warp_wait_or_abort(&a_empty[slot], (epar >> ai) & 1u, abort_flag)) break;
                    epar ^= 1u << ai;
                }
                if constexpr (ATM) {
                    // this thread's row = its TMEM lane; its 32 k fill 16 of the block's 32 columns
                    tc_fence_after();             // the MMAs that read the slot before have finished
                    const uint32_t at = tmem + ((uint32_t)(32 * (warp & 3)) << 16) + a_col0 +
                                        (uint32_t)(slot * NW * 32 + 16 * hf);
                    tmem_st16(at, o);
                    if (NW == 2) {
                        dequant_half<WT>(row + (size_t)T * raw_tile_bytes, kin & 3, hf, o);
                        tmem_st16(at + 32u, o);
                    }
                    tmem_wait_st();
                    tc_fence_before();
                } else {
                    uint8_t *at0 = a_ring + (size_t)slot * NW * 16384;
                    store_half_row(at0, m, hf, o);
                    if (NW == 2) {
                        dequant_half<WT>(row + (size_t)T * raw_tile_bytes, kin & 3, hf, o);
                        store_half_row(at0 + 16384, m, hf, o);
                    }
                    fence_proxy_async_shared();   // generic-proxy writes -> tensor core reads
                }
            } else {
                uint32_t o[32];
                dequant_regs<WT>(row, kin & 3, o);
                if (i >= p.AG) {
                    if (!warp_wait_or_abort(&a_empty[slot], (epar >> ai) & 1u, abort_flag)) break;
                    epar ^= 1u << ai;
                }
                if constexpr (ATM) {
                    // this thread's row = its TMEM lane; the 64 k of the block fill 32 columns
                    tc_fence_after();                 // the MMAs that read the slot before have finished
                    const uint32_t at = tmem + ((uint32_t)(32 * (warp & 3)) << 16) + a_col0 + (uint32_t)(slot * NW * 32);
                    tmem_st32(at, o);
                    if (NW == 2) {
                        dequant_regs<WT>(row + (size_t)T * raw_tile_bytes, kin & 3, o);
                        tmem_st32(at + 32u, o);
                    }
                    tmem_wait_st();
                    tc_fence_before();
                } else {
                    uint8_t *at0 = a_ring + (size_t)slot * NW * 16384;
                    store_row(at0, m, o);
                    if (NW == 2) {
                        dequant_regs<WT>(row + (size_t)T * raw_tile_bytes, kin & 3, o);
                        store_row(at0 + 16384, m, o);
                    }
                    fence_proxy_async_shared();       // generic-proxy writes -> tensor core reads
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&a_full[slot]);
            ai = ai + 1 == p.AG ? 0 : ai + 1;
            kin += H;
            if (kin >= kpr) {
                kin -= kpr;
                if (++rst == p.RS) { rst = 0; rpar ^= 1u; }
                new_stage = true;
            }
        }

        // ---------------- epilogue ----------------
        grid_dep_wait();                          // outputs may be read by the previous kernel
        const bool ok = warp_wait_or_abort(acc_full, 0u, abort_flag) && __all_sync(0xffffffffu, *abort_flag == 0);
        tc_fence_after();
        // The dequant warps in units of 4 (one per lane quarter): the units
        // of tile et take its batch columns in equal parts [part*cols,
        // (part+1)*cols) and add its H groups (pair: every unit a part of the
        // columns, adding the gate tile's H groups and the up tile's H groups
        // of its row).
        const int n_units = WPG * G / 4, unit = warp >> 2;
        const int upt = PAIR ? n_units : n_units / T;       // units per tile
        const int et = PAIR ? 0 : unit / upt, part = unit % upt;
        const int q = warp & 3;
        const int rloc = 32 * q + lane;           // tile row of this thread's TMEM lane
        const int row = row0 + et * kBM + rloc;
        const bool row_ok = ok && row < seg_rows;
        const bool split_k = p.ks > 1;            // partial sums: red.add, the conv runs after
        float4 cw = make_float4(0.f, 0.f, 0.f, 0.f);
        if (EPI == kTcConv && !split_k && row_ok && row < a.conv_channels)
            cw = *reinterpret_cast<const float4 *>(a.conv_w + 4 * (size_t)row);
        const int cols = p.Npad / upt;            // batch columns of this warp
        const bool conv_row = EPI == kTcConv && !split_k && row_ok && row < a.conv_channels;
        for (int c0 = part * cols; c0 < (part + 1) * cols; c0 += 8) {
            float acc[8], acc2[8];
#pragma unroll
            for (int t = 0; t < 8; ++t) acc[t] = acc2[t] = 0.f;
            if (ok) {
                // the H groups' partial sums of this tile, added in group order
                const uint32_t taddr = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)c0;
                const int g0 = et * H;
                for (int g = g0; g < g0 + H; ++g) {
                    uint32_t v[8], u[8];
                    tmem_ld8_nowait(taddr + (uint32_t)g * acc_cols, v);
                    if (NW == 2) tmem_ld8_nowait(taddr + (uint32_t)g * acc_cols + (uint32_t)p.Npad, u);
                    if (PAIR) tmem_ld8_nowait(taddr + (uint32_t)(g + H) * acc_cols, u);
                    tmem_wait_ld();
#pragma unroll
                    for (int t = 0; t < 8; ++t) {
                        acc[t] += __uint_as_float(v[t]);
                        if (NW == 2 || PAIR) acc2[t] += __uint_as_float(u[t]);
                    }
                }
            }
            if (!row_ok) continue;
            // every load of the chunk is issued before the first use
            float sc[8], cst[8][3];
#pragma unroll
            for (int t = 0; t < 8; ++t) {
                const int b = c0 + t;
                sc[t] = (a.xscale && b < a.B) ? a.xscale[b] : 1.0f;
                if (conv_row && b < a.B) {
                    const float *cs = a.conv_state + ((size_t)b * a.conv_channels + row) * 3;
                    cst[t][0] = cs[0]; cst[t][1] = cs[1]; cst[t][2] = cs[2];
                }
            }
#pragma unroll
            for (int t = 0; t < 8; ++t) {
                const int b = c0 + t;
                if (b >= a.B) continue;
                const float v = acc[t] * sc[t];
                if (EPI == kTcSwiGLU || PAIR) {
                    const float u = acc2[t] * sc[t];
                    a.dst[0][(size_t)b * a.dst_stride[0] + row] = silu(v) * u;
                } else if (EPI == kTcStore || split_k) {
                    float *d = dseg + (size_t)b * dstride + row;
                    if (split_k) atomicAdd(d, v); else *d = a.accumulate ? *d + v : v;
                } else {
                    float out = v;
                    if (conv_row) {
                        float *cs = a.conv_state + ((size_t)b * a.conv_channels + row) * 3;
                        const float accv = fmaf(cw.x, cst[t][0], fmaf(cw.y, cst[t][1], fmaf(cw.z, cst[t][2], cw.w * v)));
                        cs[0] = cst[t][1];
                        cs[1] = cst[t][2];
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
    if (warp == producer_warp) {
        // an aborted CTA may not have waited for its MMAs: wait (bounded) before freeing TMEM
        if (*abort_flag && lane == 0) mbar_wait(acc_full, 0u);
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, (uint32_t)p.tmem_cols);
    }
}

// ---------------------------------------------------------------------------
// X-stationary variant (batch up to 64 rows): CTA (chunk c, j) keeps k-chunk c
// of X resident in shared memory (one bulk copy of up to 128 KB; the producer
// of X writes it tiled, so a chunk is contiguous) and runs row tiles j,
// j + cpc, ... of that chunk, so X crosses into the SM once instead of once
// per tile. Each tile's fp32 partial sum goes to partials[c][w][b][row];
// tcx_reduce_kernel adds the chunks in order and applies the epilogue.
// 23 warps:
//   warps 0-15  dequant, set s = w / 4 takes k-blocks s*SB .. s*SB+SB-1 of
//               every raw stage (SB 256-value columns = 4*SB k-blocks) into
//               one A slot in tensor memory (one tile row per thread, its
//               TMEM lane), so one handover carries SB k-blocks;
//   warps 16-17 MMA issuers (lane 0): issuer i takes sets 2i and 2i+1 into
//               its own accumulator per tile, double-buffered across tiles
//               (one issuing thread keeps the tensor pipe about half busy at
//               N = 64; two overlap their per-MMA issue work);
//   warp 18     producer: lane 0 the raw weight stages of the CTA's tiles;
//   warps 19-22 epilogue: both issuers' accumulators (lane quarter w % 4)
//               added in issuer order -> partials, while the next tile's
//               MMAs run into the other buffers.
// ---------------------------------------------------------------------------
constexpr int kXSets = 4, kXIssuers = 2;
constexpr int kXIssuer = 4 * kXSets, kXProducer = kXIssuer + kXIssuers, kXEpi0 = kXProducer + 1;
constexpr int kXThreads = (kXEpi0 + 4) * kWarp;

struct TcxPlan {
    int NW, CB, Npad;
    int nchunk, KC, nkb;        // K chunks, values per chunk, 64-value k-blocks per chunk
    int tiles, cpc;             // row tiles over all segments, CTAs per chunk
    int seg_tiles[3], seg_off[3];
    int rows_total;
    int SB, RB, RS, spt;        // raw stages: SB 256-value columns each, spt per tile chunk
    int AG;                     // A slots per set (SB k-blocks each)
    int tmem_cols;
    uint32_t x_bytes, off_raw, off_bar;
    size_t smem;
};

template <int WT, int EPI, int KI>
__global__ void __launch_bounds__(kXThreads, 1)
tcx_gemm_kernel(const __grid_constant__ CUtensorMap tmW0, const __grid_constant__ CUtensorMap tmW1,
                const __grid_constant__ CUtensorMap tmW2, TcArgs a, TcxPlan p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    constexpr int NW = EPI == kTcSwiGLU ? 2 : 1;
    const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
    const int chunk = (int)blockIdx.x / p.cpc, j0 = (int)blockIdx.x % p.cpc;
    const int n_my = j0 < p.tiles ? (p.tiles - 1 - j0) / p.cpc + 1 : 0;

    uint8_t *x_ring = smem;                // [nkb][Npad][128 B], 128B-swizzled
    uint8_t *raw_ring = smem + p.off_raw;  // [RS][NW][128 * RB]
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + p.off_bar);
    uint64_t *raw_full = bars, *raw_empty = raw_full + p.RS;
    uint64_t *a_full = raw_empty + p.RS, *a_empty = a_full + kXSets * p.AG;
    uint64_t *x_full = a_empty + kXSets * p.AG, *acc_full = x_full + 1, *acc_empty = acc_full + 2;
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(acc_empty + 2);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);

    const uint32_t stage_bytes = (uint32_t)(kBM * p.RB);
    const uint32_t xkb_bytes = (uint32_t)(p.Npad * 128);
    constexpr int kpr = 4 * KI;                            // k-blocks per raw stage (KI == p.SB per set)
    const uint32_t acc_cols = (uint32_t)(NW * p.Npad);     // one accumulator
    // accumulator of issuer i, buffer ab: columns (2*ab + i)*acc_cols; A slot
    // (set s, i), matrix w, k-block e of the set's share: column
    // a_col0 + (((s*AG + i)*NW + w)*KI + e)*32
    const uint32_t a_col0 = 2 * kXIssuers * acc_cols;

    // tile ti of this CTA -> (segment, first row in the segment)
    auto tile_of = [&](int ti) -> int2 {
        int t = j0 + ti * p.cpc, seg = 0;
        if (a.n_seg > 1 && t >= p.seg_tiles[0]) {
            t -= p.seg_tiles[0];
            seg = 1;
            if (a.n_seg > 2 && t >= p.seg_tiles[1]) { t -= p.seg_tiles[1]; seg = 2; }
        }
        return make_int2(seg, t * kBM);
    };

    if (threadIdx.x == 0) {
        for (int i = 0; i < p.RS; ++i) { mbar_init(&raw_full[i], 1); mbar_init(&raw_empty[i], 4 * kXSets); }
        for (int i = 0; i < kXSets * p.AG; ++i) { mbar_init(&a_full[i], 4); mbar_init(&a_empty[i], 1); }
        mbar_init(x_full, 1);
        for (int i = 0; i < 2; ++i) { mbar_init(&acc_full[i], kXIssuers); mbar_init(&acc_empty[i], 4); }
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == kXProducer) tmem_alloc(tmem_holder, (uint32_t)p.tmem_cols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;
    grid_dep_launch_dependents();

    // Ring positions advance incrementally (no divisions in the loops): a
    // ring slot's fill parity flips each time the ring wraps; each A slot
    // keeps its own parity bit.
    if (warp == kXProducer) {
        if (lane == 0) {
            // weight stages (independent of the previous kernel)
            const int n_st = n_my * p.spt;
            int issued = 0, rs = 0, ti = 0, r = 0;
            uint32_t rpar = 0;
            for (int gs = 0; gs < n_st; ++gs) {
                if (gs >= p.RS && !wait_or_abort(&raw_empty[rs], rpar ^ 1u, abort_flag)) break;
                const int2 sr = tile_of(ti);
                const CUtensorMap *tmA = sr.x == 0 ? &tmW0 : (sr.x == 1 ? &tmW1 : &tmW2);
                mbar_arrive_expect_tx(&raw_full[rs], (uint32_t)NW * stage_bytes);
                uint8_t *dst = raw_ring + (size_t)rs * NW * stage_bytes;
                const int xcol = (chunk * p.spt + r) * (p.RB / 4);
                tma_load_2d(dst, tmA, xcol, sr.y, &raw_full[rs]);
                if (NW == 2) tma_load_2d(dst + stage_bytes, &tmW1, xcol, sr.y, &raw_full[rs]);
                issued = gs + 1;
                if (++r == p.spt) { r = 0; ++ti; }
                if (++rs == p.RS) { rs = 0; rpar ^= 1u; }
            }
            // drain: every copy issued has landed before the CTA exits
            for (int gs = issued - p.RS < 0 ? 0 : issued - p.RS; gs < issued; ++gs)
                mbar_wait(&raw_full[gs % p.RS], (uint32_t)((gs / p.RS) & 1));
        }
    } else if (warp >= kXIssuer && warp < kXIssuer + kXIssuers) {
        // MMA issue is serial in the issuing thread, so the loop keeps the
        // work between MMAs to a minimum: descriptors advance by constants.
        const int ii = warp - kXIssuer;
        if (lane == 0 && n_my > 0) {
            const uint32_t idesc = idesc_f16(p.Npad);
            const uint64_t xdesc0 = sw128_desc(smem_addr(x_ring));
            const uint32_t xstep = xkb_bytes >> 4;     // descriptor units per k-block
            int sl[2] = {0, 0};          // next A slot of each of this issuer's sets
            uint32_t fpar[2] = {0, 0};   // a_full parity bit per slot
            bool ok = wait_or_abort(x_full, 0u, abort_flag);
            for (int ti = 0; ok && ti < n_my; ++ti) {
                const int ab = ti & 1;
                if (ti >= 2 && !wait_or_abort(&acc_empty[ab], (uint32_t)(((ti >> 1) - 1) & 1), abort_flag)) break;
                const uint32_t d_tmem = tmem + (uint32_t)(2 * ab + ii) * acc_cols;
                for (int st = 0; ok && st < p.spt; ++st) {
#pragma unroll
                    for (int s2 = 0; s2 < 2; ++s2) {
                        const int s = 2 * ii + s2;
                        const int kb0 = st * kpr + s * KI, slot = s * p.AG + sl[s2];
                        if (!wait_or_abort(&a_full[slot], (fpar[s2] >> sl[s2]) & 1u, abort_flag)) { ok = false; break; }
                        fpar[s2] ^= 1u << sl[s2];
                        tc_fence_after();
                        const uint64_t bd = xdesc0 + (uint64_t)(kb0 * xstep);
                        const uint32_t at = tmem + a_col0 + (uint32_t)(slot * NW * KI * 32);
                        // this issuer's first MMA of the tile (per matrix) overwrites its accumulator
                        const uint32_t acc0 = (st > 0 || s2 > 0) ? 1u : 0u;
#pragma unroll
                        for (int e = 0; e < KI; ++e)
#pragma unroll
                            for (int w = 0; w < NW; ++w)
#pragma unroll
                                for (int jj = 0; jj < 4; ++jj)
                                    umma_f16_ta(d_tmem + (uint32_t)(w * p.Npad), at + (uint32_t)((w * KI + e) * 32 + 8 * jj),
                                                bd + (uint64_t)(e * xstep + 2 * jj), idesc, (e > 0 || jj > 0) ? 1u : acc0);
                        umma_commit(&a_empty[slot]);
                        sl[s2] = sl[s2] + 1 == p.AG ? 0 : sl[s2] + 1;
                    }
                }
                if (ok) umma_commit(&acc_full[ab]);
            }
        }
    } else if (warp < kXIssuer) {
        // ---------------- dequant ----------------
        // every raw stage holds this set's share (KI k-blocks), one A slot per stage
        const int s = warp >> 2, q = warp & 3;
        const int m = 32 * q + lane;
        const uint32_t lane_addr = tmem + ((uint32_t)(32 * q) << 16);
        int sl = 0, rs = 0;
        uint32_t epar = 0, rpar = 0;   // a_empty parity bit per slot; raw ring fill parity
        bool ok = true;
        const int n_st = n_my * p.spt;
        for (int gs = 0; ok && gs < n_st; ++gs) {
            if (!warp_wait_or_abort(&raw_full[rs], rpar, abort_flag)) break;
            const uint8_t *stg = raw_ring + (size_t)rs * NW * stage_bytes + (size_t)m * p.RB;
            const int slot = s * p.AG + sl;
            const uint32_t at = lane_addr + a_col0 + (uint32_t)(slot * NW * KI * 32);
            for (int e = 0; e < KI; ++e) {
                const int sub = s * KI + e;   // k-block within the stage
                const uint8_t *row = stg + (size_t)(sub >> 2) * p.CB;
                uint32_t o[32], o2[32];
                dequant_regs<WT>(row, sub & 3, o);
                if (NW == 2) dequant_regs<WT>(row + stage_bytes, sub & 3, o2);
                if (e == KI - 1) {   // this warp's rows of the stage are read
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&raw_empty[rs]);
                }
                if (e == 0) {
                    if (gs >= p.AG) {
                        if (!warp_wait_or_abort(&a_empty[slot], (epar >> sl) & 1u, abort_flag)) { ok = false; break; }
                        epar ^= 1u << sl;
                    }
                    tc_fence_after();
                }
                tmem_st32(at + (uint32_t)(e * 32), o);
                if (NW == 2) tmem_st32(at + (uint32_t)((KI + e) * 32), o2);
            }
            if (!ok) break;
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&a_full[slot]);
            sl = sl + 1 == p.AG ? 0 : sl + 1;
            if (++rs == p.RS) { rs = 0; rpar ^= 1u; }
        }
    } else {
        // ---------------- epilogue: accumulators -> partials ----------------
        const int q = warp & 3;
        grid_dep_wait();   // the partials may still be read by the previous kernel
        // The X chunk (written by the previous kernel) comes from here, not
        // from the producer warp: a divergent lane of that warp waiting for
        // the previous kernel would hold back its weight stages.
        const bool x_issuer = warp == kXEpi0 && lane == 0 && n_my > 0;
        if (x_issuer) {
            mbar_arrive_expect_tx(x_full, p.x_bytes);
            bulk_g2s(x_ring, reinterpret_cast<const uint8_t *>(a.X16) + (size_t)chunk * p.x_bytes, p.x_bytes, x_full);
        }
        const uint32_t lane_addr = tmem + ((uint32_t)(32 * q) << 16);
        for (int ti = 0; ti < n_my; ++ti) {
            const int ab = ti & 1;
            if (!warp_wait_or_abort(&acc_full[ab], (uint32_t)((ti >> 1) & 1), abort_flag)) break;
            tc_fence_after();
            const int2 sr = tile_of(ti);
            const int seg = sr.x, row0 = sr.y;
            const int grow0 = (seg == 0 ? p.seg_off[0] : seg == 1 ? p.seg_off[1] : p.seg_off[2]) + row0;
            const int seg_rows = seg == 0 ? a.seg_rows[0] : (seg == 1 ? a.seg_rows[1] : a.seg_rows[2]);
            const bool row_ok = row0 + 32 * q + lane < seg_rows;
            const size_t grow = (size_t)grow0 + 32 * q + lane;
            const uint32_t acc0 = lane_addr + (uint32_t)(2 * ab) * acc_cols;   // issuer 0; issuer 1 follows
#pragma unroll
            for (int w = 0; w < NW; ++w) {
                float *pw = a.partials + (size_t)(chunk * NW + w) * a.B * p.rows_total + grow;
                for (int c0 = 0; c0 < p.Npad; c0 += 32) {
                    uint32_t v[32], u[32];
                    tmem_ld32_nowait(acc0 + (uint32_t)(w * p.Npad + c0), v);
                    tmem_ld32_nowait(acc0 + acc_cols + (uint32_t)(w * p.Npad + c0), u);
                    tmem_wait_ld();
                    if (row_ok) {
#pragma unroll
                        for (int t = 0; t < 32; ++t)
                            if (c0 + t < a.B)
                                pw[(size_t)(c0 + t) * p.rows_total] = __uint_as_float(v[t]) + __uint_as_float(u[t]);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[ab]);
        }
        if (x_issuer) mbar_wait(x_full, 0u);   // the copy has landed before the CTA exits
    }

    if (*abort_flag && threadIdx.x == 0) atomicExch(&g_device_error, LI_ERR_TIMEOUT);
    tc_fence_before();
    __syncthreads();
    if (warp == kXProducer) {
        // an aborted CTA may have MMAs in flight: wait (bounded) for the last commits
        if (*abort_flag && lane == 0 && n_my > 0) {
            mbar_wait(&acc_full[(n_my - 1) & 1], (uint32_t)(((n_my - 1) >> 1) & 1));
        }
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, (uint32_t)p.tmem_cols);
    }
}

// The chunks' partial sums added in chunk order, scaled by the X row scale,
// then the epilogue; four consecutive rows per thread.
template <int EPI>
__global__ void __launch_bounds__(256) tcx_reduce_kernel(TcArgs a, int nchunk, int rows_total, int seg_off1,
                                                         int seg_off2) {
    constexpr int NW = EPI == kTcSwiGLU ? 2 : 1;
    grid_dep_wait();
    grid_dep_launch_dependents();
    const int nq = rows_total / 4;
    const int it = (int)blockIdx.x * 256 + (int)threadIdx.x;
    if (it >= a.B * nq) return;
    const int b = it / nq, gr = 4 * (it % nq);
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f), u = v;
    for (int c = 0; c < nchunk; ++c) {
        const float4 t = *reinterpret_cast<const float4 *>(a.partials + ((size_t)(c * NW) * a.B + b) * rows_total + gr);
        v.x += t.x; v.y += t.y; v.z += t.z; v.w += t.w;
        if (NW == 2) {
            const float4 t2 =
                *reinterpret_cast<const float4 *>(a.partials + ((size_t)(c * NW + 1) * a.B + b) * rows_total + gr);
            u.x += t2.x; u.y += t2.y; u.z += t2.z; u.w += t2.w;
        }
    }
    const float sc = a.xscale ? a.xscale[b] : 1.0f;
    float r[4] = {v.x * sc, v.y * sc, v.z * sc, v.w * sc};
    const int seg = gr >= seg_off2 && a.n_seg > 2 ? 2 : (gr >= seg_off1 && a.n_seg > 1 ? 1 : 0);
    const int row = gr - (seg == 0 ? 0 : seg == 1 ? seg_off1 : seg_off2);
    float *dst = (seg == 0 ? a.dst[0] : seg == 1 ? a.dst[1] : a.dst[2]) +
                 (size_t)b * (seg == 0 ? a.dst_stride[0] : seg == 1 ? a.dst_stride[1] : a.dst_stride[2]) + row;
    if (EPI == kTcSwiGLU) {
        const float g[4] = {u.x * sc, u.y * sc, u.z * sc, u.w * sc};
#pragma unroll
        for (int e = 0; e < 4; ++e) r[e] = silu(r[e]) * g[e];
    } else if (EPI == kTcConv && row < a.conv_channels) {
        // rows row .. row+3 are all conv channels (conv_channels is a multiple of 4)
        float *cs = a.conv_state + ((size_t)b * a.conv_channels + row) * 3;
        float4 s4[3];
#pragma unroll
        for (int e = 0; e < 3; ++e) s4[e] = reinterpret_cast<const float4 *>(cs)[e];
        const float st[12] = {s4[0].x, s4[0].y, s4[0].z, s4[0].w, s4[1].x, s4[1].y,
                              s4[1].z, s4[1].w, s4[2].x, s4[2].y, s4[2].z, s4[2].w};
        float ns[12];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float4 cw = *reinterpret_cast<const float4 *>(a.conv_w + 4 * (size_t)(row + e));
            const float x = r[e];
            const float acc = fmaf(cw.x, st[3 * e], fmaf(cw.y, st[3 * e + 1], fmaf(cw.z, st[3 * e + 2], cw.w * x)));
            ns[3 * e] = st[3 * e + 1];
            ns[3 * e + 1] = st[3 * e + 2];
            ns[3 * e + 2] = x;
            r[e] = silu(acc);
        }
#pragma unroll
        for (int e = 0; e < 3; ++e)
            reinterpret_cast<float4 *>(cs)[e] = make_float4(ns[4 * e], ns[4 * e + 1], ns[4 * e + 2], ns[4 * e + 3]);
    }
    if (EPI == kTcStore && a.accumulate) {
        const float4 o = *reinterpret_cast<const float4 *>(dst);
        r[0] = o.x + r[0]; r[1] = o.y + r[1]; r[2] = o.z + r[2]; r[3] = o.w + r[3];
    }
    *reinterpret_cast<float4 *>(dst) = make_float4(r[0], r[1], r[2], r[3]);
}

// The conv epilogue of a K-split in-projection: the split CTAs have added
// their partial sums into dst[0] (raw projections, row scale applied); the
// first conv_channels columns of every row go through the causal conv1d
// (the tap order and arithmetic of the in-kernel epilogue) and SiLU, in place,
// and the conv state shifts. One (row, channel) per thread.
__global__ void __launch_bounds__(256) tc_conv_finish_kernel(TcArgs a) {
    grid_dep_wait();
    grid_dep_launch_dependents();
    const int64_t it = (int64_t)blockIdx.x * 256 + threadIdx.x;
    if (it >= (int64_t)a.B * a.conv_channels) return;
    const int b = (int)(it / a.conv_channels), c = (int)(it % a.conv_channels);
    float *d = a.dst[0] + (size_t)b * a.dst_stride[0] + c;
    float *cs = a.conv_state + ((size_t)b * a.conv_channels + c) * 3;
    const float v = *d;
    const float c0 = cs[0], c1 = cs[1], c2 = cs[2];
    const float *w = a.conv_w + 4 * (size_t)c;
    const float acc = fmaf(w[0], c0, fmaf(w[1], c1, fmaf(w[2], c2, w[3] * v)));
    cs[0] = c1;
    cs[1] = c2;
    cs[2] = v;
    *d = silu(acc);
}

// ---------------------------------------------------------------------------
// x -> f16 with optional RMSNorm and a per-row power-of-two scale
// ---------------------------------------------------------------------------
// NV > 0: the row's K/4 float4 words (at most 256*NV) are loaded once, all
// before the first reduction, and kept in registers for the conversion (one
// memory round trip per row instead of two dependent passes); NV = 0 re-reads
// x in a second pass for longer rows. Both give the same bits: every thread
// visits its words in the same order either way.
template <int NV>
__global__ void __launch_bounds__(256)
tc_prep_kernel(const float *__restrict__ x, int x_stride, const float *__restrict__ gamma, float eps, int K,
               __half *__restrict__ X16, float *__restrict__ xscale, int x_npad, int early_dependents) {
    __shared__ float s_sq[8], s_mx[8];
    const int b = blockIdx.x, t = threadIdx.x, n4 = K / 4;
    // An X-stationary GEMM after this kernel may launch at once: it streams
    // its weights meanwhile and waits for this kernel before it reads X16.
    if (early_dependents) grid_dep_launch_dependents();
    grid_dep_wait();
    const float4 *x4 = reinterpret_cast<const float4 *>(x + (size_t)b * x_stride);
    const float4 *g4 = reinterpret_cast<const float4 *>(gamma);
    float sq = 0.f, mx = 0.f;
    float4 vg[NV > 0 ? NV : 1];           // x * gamma of this thread's words
    if constexpr (NV > 0) {
        float4 v[NV];
#pragma unroll
        for (int j = 0; j < NV; ++j)
            if (t + 256 * j < n4) v[j] = x4[t + 256 * j];
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            if (t + 256 * j >= n4) break;
            sq = fmaf(v[j].x, v[j].x, fmaf(v[j].y, v[j].y, fmaf(v[j].z, v[j].z, fmaf(v[j].w, v[j].w, sq))));
            const float4 g = gamma ? g4[t + 256 * j] : make_float4(1.f, 1.f, 1.f, 1.f);
            vg[j] = make_float4(v[j].x * g.x, v[j].y * g.y, v[j].z * g.z, v[j].w * g.w);
            mx = fmaxf(mx, fmaxf(fmaxf(fabsf(vg[j].x), fabsf(vg[j].y)), fmaxf(fabsf(vg[j].z), fabsf(vg[j].w))));
        }
    } else {
        for (int i = t; i < n4; i += 256) {
            const float4 v = x4[i];
            sq = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, sq))));
            float4 g = gamma ? g4[i] : make_float4(1.f, 1.f, 1.f, 1.f);
            mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x * g.x), fabsf(v.y * g.y)), fmaxf(fabsf(v.z * g.z), fabsf(v.w * g.w))));
        }
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
    auto put = [&](int i, float4 w) {
        const __half2 lo = __floats2half2_rn(w.x * inv, w.y * inv);
        const __half2 hi = __floats2half2_rn(w.z * inv, w.w * inv);
        // four consecutive k stay together in either layout (8 bytes)
        __half *dst = X16 + (x_npad ? tiled_x_offset(b, 4 * i, x_npad) : (size_t)b * K + 4 * i);
        *reinterpret_cast<uint2 *>(dst) = make_uint2(*reinterpret_cast<const uint32_t *>(&lo),
                                                     *reinterpret_cast<const uint32_t *>(&hi));
    };
    if constexpr (NV > 0) {
#pragma unroll
        for (int j = 0; j < NV; ++j)
            if (t + 256 * j < n4) put(t + 256 * j, vg[j]);
    } else {
        for (int i = t; i < n4; i += 256) {
            const float4 v = x4[i];
            const float4 g = gamma ? g4[i] : make_float4(1.f, 1.f, 1.f, 1.f);
            put(i, make_float4(v.x * g.x, v.y * g.y, v.z * g.z, v.w * g.w));
        }
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

// Columns per raw stage to try first. One 256-value column per stage (18 KB
// of Q4_K rows) with four stages and two 32 KB X slots measured best for the
// DeltaNet layer step at 64 sequences (B200, chained graph: 87.0 us vs 93.4
// with two-column stages; the kernels alone take the same time, the
// smaller footprint overlaps better with its neighbours), and is neutral for
// the 64-row SwiGLU FFN (70.4 vs 71.2 us).
int tc_default_sb() { return 1; }

int plan(const TcArgs &a, TcPlan *p) {
    if (a.wtype != LI_WTYPE_Q4_K && a.wtype != LI_WTYPE_Q8_0) return LI_ERR_UNSUPPORTED;
    if (a.K <= 0 || a.K % 256 || a.B <= 0 || a.B > 256) return LI_ERR_BAD_SHAPE;
    p->CB = a.wtype == LI_WTYPE_Q4_K ? 144 : 272;
    p->Npad = (a.B + 31) / 32 * 32;
    if (p->Npad > 512) return LI_ERR_BAD_SHAPE;
    int seg_tiles_total = 0;
    for (int s = 0; s < 3; ++s) {
        p->seg_tiles[s] = s < a.n_seg ? (a.seg_rows[s] + kBM - 1) / kBM : 0;
        seg_tiles_total += p->seg_tiles[s];
    }
    int sms = 148;
    {
        int dev = 0;
        if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    }
    const int cols256 = a.K / 256;
    const size_t x_b = (size_t)p->Npad * 128;
    // Two 128-row tiles per CTA first (T = 2: every X k-block in shared
    // memory feeds both tiles, which halves the X bytes per weight byte; one
    // weight matrix and one segment only), then one. A in tensor memory first
    // (the dequantized tile never touches shared memory, which leaves the
    // shared-memory bandwidth to the raw blocks and X), with as many groups
    // as the TMEM holds (each group: N accumulator columns and 32 columns per
    // A slot, per weight matrix); A in shared memory when the accumulators
    // leave no room. Then raw stages of SB columns, then K splits so that the
    // CTAs cover the SMs (a CTA streams its weights at a limited rate: 97
    // CTAs moving the 28.5 MB in-projection with nothing else to do take 8.3
    // us, measured on B200; the partial sums meet in fp32 reductions into a
    // zeroed output, and the conv epilogue then runs in tc_conv_finish_kernel),
    // then the deepest rings that fit.
    // {raw stages, A slots per group, k-blocks per group per X slot, X slots}
    static const int kRings1[][4] = {{4, 2, 1, 2}, {4, 2, 2, 2}, {3, 2, 2, 2}, {2, 2, 2, 2}, {3, 2, 1, 2},
                                     {2, 2, 1, 2}, {3, 1, 2, 2}, {2, 1, 2, 2}, {3, 1, 1, 2}, {2, 1, 1, 2},
                                     {2, 1, 1, 1}};
    static const int kRings2[][4] = {{4, 2, 2, 2}, {3, 2, 2, 2}, {2, 2, 2, 2}, {4, 2, 1, 2}, {3, 2, 1, 2},
                                     {2, 2, 1, 2}, {2, 1, 2, 2}, {2, 1, 1, 2}, {2, 1, 1, 1}};
    // eight dequant warps per group (at most two groups): the tensor memory
    // left by two groups' accumulators holds four A slots per group, so the
    // dequant runs up to four k-blocks ahead of the MMAs. Preferred from 128
    // batch columns; below, four warps in four groups (measured on B200,
    // Q4_K: SwiGLU FFN 4096 -> 12288 -> 4096 at 256 rows 133.6 us against
    // 155.2; at 64 rows 86.9 against 64.2; DeltaNet layer step at 64
    // sequences 98.7 against 86.3, at 128 sequences 157.9 against 159.2)
    static const int kRings8[][4] = {{6, 4, 1, 4}, {6, 4, 1, 2}, {4, 4, 1, 4}, {4, 4, 1, 2}, {4, 3, 1, 2},
                                     {3, 4, 1, 2}, {2, 4, 1, 2}, {3, 3, 1, 2}, {2, 2, 1, 2}};
    // SwiGLU: the gate/up tile pair first (one accumulator per group, so
    // twice the groups of the two-matrix tile fit in the tensor memory:
    // measured on B200 at 64 rows, 4096 -> 12288, 39.5 us against 41.0 with
    // both matrices in every tile)
    for (int T = a.epi == kTcSwiGLU ? 2 : kMaxTilesPerCta; T >= 1; --T) {
        const bool pair = a.epi == kTcSwiGLU && T == 2;
        if (T > 1 && !pair && (a.n_seg != 1 || a.epi == kTcSwiGLU || seg_tiles_total < 2)) continue;
        p->pair = pair ? 1 : 0;
        p->NW = a.epi == kTcSwiGLU && !pair ? 2 : 1;
        p->tiles = pair ? 2 * p->seg_tiles[0] : seg_tiles_total;
        const int nwn = p->NW * p->Npad;                  // TMEM columns per group
        const size_t a_b = (size_t)p->NW * 16384;         // one A slot (shared memory)
        if (nwn > 512) continue;
        const int n_groups = (p->tiles + T - 1) / T;     // tile groups (CTAs per K split)
        for (int wpg : {p->Npad >= 128 ? 8 : 4, p->Npad >= 128 ? 4 : 8})
        for (int atm = 1; atm >= 0; --atm) {
            for (int G = wpg == 8 ? 2 : kMaxGroups; G >= T; G /= 2) {
                if (G * nwn > 512 || ((wpg + 1) * G + 2) * kWarp > kMaxThreads) continue;
                const int H = G / T;
                p->G = G; p->T = T; p->H = H;
                p->WPG = wpg;
                p->atm = atm;
                for (int sb : {tc_default_sb(), 1, 2}) {
                    if (sb < 1 || cols256 % sb || p->CB * sb / 4 > 256 || (4 * sb) % H) continue;
                    p->SB = sb;
                    p->RB = sb * p->CB;
                    p->n_raw = cols256 / sb;
                    p->ks = 1;
                    if (a.epi == kTcStore || a.epi == kTcConv)
                        while ((p->ks + 1) * n_groups <= sms && p->n_raw / (p->ks + 1) >= 2) ++p->ks;
                    const int kpr = 4 * sb;
                    const size_t raw_b = (size_t)p->NW * T * kBM * p->RB;
                    const int n_rings = wpg == 8 ? (int)(sizeof(kRings8) / sizeof(kRings8[0]))
                                        : T == 2 ? (int)(sizeof(kRings2) / sizeof(kRings2[0]))
                                                 : (int)(sizeof(kRings1) / sizeof(kRings1[0]));
                    for (int ri = 0; ri < n_rings; ++ri) {
                        const int *rg = wpg == 8 ? kRings8[ri] : T == 2 ? kRings2[ri] : kRings1[ri];
                        const int rs = rg[0], ag = rg[1], xm = rg[2], xs = rg[3];
                        if (kpr % (H * xm)) continue;     // X slots tile every CTA's k-blocks
                        const int tcols = G * nwn + (atm ? G * ag * p->NW * 32 : 0);
                        if (tcols > 512) continue;
                        int cols = 32;
                        while (cols < tcols) cols <<= 1;
                        p->tmem_cols = cols;
                        p->RS = rs; p->AG = ag; p->XM = xm; p->XS = xs;
                        p->off_a = 0;
                        p->off_x = atm ? 0u : (uint32_t)(G * ag * a_b);
                        p->off_raw = p->off_x + (uint32_t)((size_t)xs * H * xm * x_b);
                        p->off_bar = p->off_raw + (uint32_t)(rs * raw_b);
                        p->smem = p->off_bar + 8 * (2 * rs + 2 * G * ag + 2 * xs + 1) + 16 + 1024;
                        if (p->smem <= (size_t)kMaxSmem) return 0;
                    }
                }
            }
        }
    }
    return LI_ERR_BAD_SHAPE;
}

// X-stationary plan: needs partials (unless sizing), batch <= 32, rows and
// strides in multiples of 4 (the reduce kernel moves four rows at a time).
// X chunks of 64 KB come first: they leave room for 4 raw stages (a stage's
// load then overlaps the dequant of the ones before it) and give 2x the
// (tile, chunk) items to spread over the SMs (layer step at hidden 4096, B =
// 3-32: 3-3.5 us faster than with 128 KB chunks and 2-3 raw stages).
// Measured on B200 (DeltaNet layer step, hidden 4096): 3-32 rows gain (8
// rows 54 us vs 58, 3 rows 48 vs 52); at 64 rows the K split's partial sums
// and their reduce cost more than the shorter X stream saves (112 us vs 105).
constexpr int kTcxMaxRows = 32;

int planx(const TcArgs &a, TcxPlan *p, bool sizing) {
    if (a.wtype != LI_WTYPE_Q4_K && a.wtype != LI_WTYPE_Q8_0) return LI_ERR_UNSUPPORTED;
    if (a.K <= 0 || a.K % 256 || a.B <= 0 || a.B > kTcxMaxRows || a.n_seg < 1 || a.n_seg > 3) return LI_ERR_BAD_SHAPE;
    if (a.epi == kTcSwiGLU && a.n_seg != 1) return LI_ERR_BAD_SHAPE;
    p->NW = a.epi == kTcSwiGLU ? 2 : 1;
    p->CB = a.wtype == LI_WTYPE_Q4_K ? 144 : 272;
    p->Npad = (a.B + 31) / 32 * 32;
    p->tiles = 0;
    p->rows_total = 0;
    for (int s = 0; s < 3; ++s) {
        const int rows = s < a.n_seg ? a.seg_rows[s] : 0;
        if (rows % 4) return LI_ERR_BAD_SHAPE;
        p->seg_off[s] = p->rows_total;
        p->seg_tiles[s] = (rows + kBM - 1) / kBM;
        p->tiles += p->seg_tiles[s];
        p->rows_total += rows;
    }
    if (!sizing) {
        if (!a.partials || !aligned16(a.partials) || !aligned16(a.X16)) return LI_ERR_MISALIGNED;
        for (int s = 0; s < a.n_seg; ++s)
            if (a.dst_stride[s] % 4 || !aligned16(a.dst[s])) return LI_ERR_MISALIGNED;
        if (a.epi == kTcConv && (a.conv_channels % 4 || !aligned16(a.conv_state) || !aligned16(a.conv_w)))
            return LI_ERR_MISALIGNED;
    }
    int sms = 148;
    {
        int dev = 0;
        if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    }
    for (int xb : {64 * 1024, 128 * 1024}) {
        int kc = a.K;
        while (kc > 256 && ((size_t)p->Npad * kc * 2 > (size_t)xb || a.K % kc || kc % 256)) kc -= 256;
        if ((size_t)p->Npad * kc * 2 > (size_t)xb || a.K % kc) continue;
        p->KC = kc;
        p->nchunk = a.K / kc;
        p->nkb = kc / 64;
        if (p->nkb > 4 * 256 || p->nkb % 4) continue;
        p->x_bytes = (uint32_t)((size_t)p->Npad * kc * 2);
        for (int sb : {2, 1}) {
            if ((kc / 256) % sb) continue;
            // TMEM: two accumulator buffers, then 4 sets x AG slots of SB k-blocks per matrix
            const int accs = 2 * kXIssuers * p->NW * p->Npad;   // two buffers per issuer
            const int ag = accs + 4 * 2 * p->NW * sb * 32 <= 512 ? 2 : 1;
            const int tcols = accs + 4 * ag * p->NW * sb * 32;
            if (tcols > 512) continue;
            p->AG = ag;
            p->tmem_cols = 32;
            while (p->tmem_cols < tcols) p->tmem_cols <<= 1;
            p->SB = sb;
            p->RB = sb * p->CB;
            p->spt = kc / (256 * sb);
            const size_t stage = (size_t)p->NW * kBM * p->RB;
            for (int rs : {4, 3, 2}) {
                p->RS = rs;
                p->off_raw = (p->x_bytes + 1023u) / 1024u * 1024u;
                p->off_bar = p->off_raw + (uint32_t)(rs * stage);
                p->smem = p->off_bar + 8 * (2 * rs + 2 * 4 * ag + 1 + 4) + 16 + 1024;
                if (p->smem <= (size_t)kMaxSmem) {
                    p->cpc = sms / p->nchunk;
                    if (p->cpc < 1) p->cpc = 1;
                    if (p->cpc > p->tiles) p->cpc = p->tiles;
                    return 0;
                }
            }
        }
    }
    return LI_ERR_BAD_SHAPE;
}

template <int WT, int EPI, int KI>
int launch_x(const CUtensorMap *maps, const TcArgs &a, const TcxPlan &p, cudaStream_t stream, bool pdl) {
    auto kern = tcx_gemm_kernel<WT, EPI, KI>;
    static std::once_flag once;
    static cudaError_t attr_err = cudaSuccess;
    std::call_once(once, [&] {
        attr_err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem);
    });
    if (attr_err != cudaSuccess) return (int)attr_err;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(p.nchunk * p.cpc));
    cfg.blockDim = dim3((unsigned)kXThreads);
    cfg.dynamicSmemBytes = p.smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, maps[0], maps[1], maps[2], a, p);
    if (e != cudaSuccess) return (int)e;
    const int items = a.B * (p.rows_total / 4);
    return (int)launch_pdl(tcx_reduce_kernel<EPI>, dim3((unsigned)((items + 255) / 256)), dim3(256), 0, stream, true,
                           a, p.nchunk, p.rows_total, p.seg_off[1], p.seg_off[2]);
}

template <int WT, int EPI>
int launch_x(const CUtensorMap *maps, const TcArgs &a, const TcxPlan &p, cudaStream_t stream, bool pdl) {
    return p.SB == 2 ? launch_x<WT, EPI, 2>(maps, a, p, stream, pdl) : launch_x<WT, EPI, 1>(maps, a, p, stream, pdl);
}

template <int WT, int EPI, bool ATM, int WPG>
int launch_kernel(const CUtensorMap *maps, const TcArgs &a, const TcPlan &p, cudaStream_t stream, bool pdl) {
    auto kern = tc_gemm_kernel<WT, EPI, ATM, WPG>;
    static std::once_flag once;
    static cudaError_t attr_err = cudaSuccess;
    std::call_once(once, [&] {
        attr_err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem);
    });
    if (attr_err != cudaSuccess) return (int)attr_err;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((p.tiles + p.T - 1) / p.T * p.ks));
    cfg.blockDim = dim3((unsigned)(((WPG + 1) * p.G + 2) * kWarp));
    cfg.dynamicSmemBytes = p.smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, maps[0], maps[1], maps[2], a, p);
    if (e != cudaSuccess || EPI != kTcConv || p.ks == 1) return (int)e;
    const int64_t items = (int64_t)a.B * a.conv_channels;
    return (int)launch_pdl(tc_conv_finish_kernel, dim3((unsigned)((items + 255) / 256)), dim3(256), 0, stream, true,
                           a);
}

template <int WT, int EPI>
int launch_kernel(const CUtensorMap *maps, const TcArgs &a, const TcPlan &p, cudaStream_t stream, bool pdl) {
    if (p.WPG == 8)
        return p.atm ? launch_kernel<WT, EPI, true, 8>(maps, a, p, stream, pdl)
                     : launch_kernel<WT, EPI, false, 8>(maps, a, p, stream, pdl);
    return p.atm ? launch_kernel<WT, EPI, true, 4>(maps, a, p, stream, pdl)
                 : launch_kernel<WT, EPI, false, 4>(maps, a, p, stream, pdl);
}

}  // namespace

int tc_prep_launch(const float *x, int x_stride, const float *gamma, float eps, int B, int K, __half *X16,
                   float *xscale, cudaStream_t stream, bool pdl, int x_npad, bool early_dependents) {
    if (K % 8 || !aligned16(x) || (gamma && !aligned16(gamma)) || !aligned16(X16)) return LI_ERR_MISALIGNED;
    if (x_npad && (x_npad < B || x_npad % 8 || K % 64)) return LI_ERR_BAD_SHAPE;
    const int nv = (K / 4 + 255) / 256;   // float4 words per thread
    const dim3 grid((unsigned)B), block(256);
    if (nv <= 4)
        return (int)launch_pdl(tc_prep_kernel<4>, grid, block, 0, stream, pdl, x, x_stride, gamma, eps, K, X16, xscale,
                               x_npad, (int)early_dependents);
    if (nv <= 8)
        return (int)launch_pdl(tc_prep_kernel<8>, grid, block, 0, stream, pdl, x, x_stride, gamma, eps, K, X16, xscale,
                               x_npad, (int)early_dependents);
    if (nv <= 12)
        return (int)launch_pdl(tc_prep_kernel<12>, grid, block, 0, stream, pdl, x, x_stride, gamma, eps, K, X16,
                               xscale, x_npad, (int)early_dependents);
    if (nv <= 20)
        return (int)launch_pdl(tc_prep_kernel<20>, grid, block, 0, stream, pdl, x, x_stride, gamma, eps, K, X16,
                               xscale, x_npad, (int)early_dependents);
    return (int)launch_pdl(tc_prep_kernel<0>, grid, block, 0, stream, pdl, x, x_stride, gamma, eps, K, X16, xscale,
                           x_npad, (int)early_dependents);
}

bool tc_gemm_splits_k(const TcArgs &a) {
    TcArgs c = a;
    if (!c.X16) c.X16 = reinterpret_cast<const __half *>(c.partials);
    TcxPlan px;
    if (planx(c, &px, false) == 0) return false;   // the X-stationary kernel stores whole sums
    TcPlan p;
    return plan(a, &p) == 0 && p.ks > 1;
}

bool tc_gemm_x_stationary(const TcArgs &a) {
    TcArgs c = a;
    if (!c.X16) c.X16 = reinterpret_cast<const __half *>(c.partials);
    TcxPlan px;
    return planx(c, &px, false) == 0;
}

int tc_gemm_x_npad(const TcArgs &a) {
    TcArgs c = a;
    if (!c.X16) c.X16 = reinterpret_cast<const __half *>(c.partials);   // alignment of a pointer to come
    TcxPlan px;
    if (planx(c, &px, false) == 0) return px.Npad;
    TcPlan p;
    return plan(c, &p) == 0 ? p.Npad : 0;
}

size_t tc_gemm_partials_bytes(int wtype, int epi, int K, int rows_total, int B) {
    TcArgs a = {};
    a.wtype = wtype; a.epi = epi; a.K = K; a.total_rows = rows_total; a.B = B;
    a.n_seg = 1; a.seg_rows[0] = rows_total;
    TcxPlan p;
    if (planx(a, &p, true)) return 0;
    return (size_t)p.nchunk * p.NW * B * p.rows_total * sizeof(float);
}

namespace {
int launch_tcx(const TcArgs &a, const TcxPlan &p, cudaStream_t stream, bool pdl) {
    const size_t rb = li_row_bytes(a.wtype, a.K);
    CUtensorMap maps[4];
    memset(maps, 0, sizeof(maps));
    int rc;
    const int nw = a.epi == kTcSwiGLU ? 2 : a.n_seg;
    for (int s = 0; s < 3; ++s) {
        const int src = s < nw ? s : 0;
        const int rows = a.epi == kTcSwiGLU ? a.seg_rows[0] : a.seg_rows[src];
        if (!aligned16(a.W[src])) return LI_ERR_MISALIGNED;
        rc = encode_2d(&maps[s], CU_TENSOR_MAP_DATA_TYPE_UINT32, a.W[src], rb / 4, (uint64_t)rows, rb,
                       (uint32_t)(p.RB / 4), kBM, CU_TENSOR_MAP_SWIZZLE_NONE);
        if (rc) return rc;
    }
    if (!aligned16(a.X16)) return LI_ERR_MISALIGNED;   // X comes by one bulk copy (no tensor map)
    const bool q4 = a.wtype == LI_WTYPE_Q4_K;
    switch (a.epi) {
    case kTcStore: return q4 ? launch_x<LI_WTYPE_Q4_K, kTcStore>(maps, a, p, stream, pdl)
                              : launch_x<LI_WTYPE_Q8_0, kTcStore>(maps, a, p, stream, pdl);
    case kTcSwiGLU: return q4 ? launch_x<LI_WTYPE_Q4_K, kTcSwiGLU>(maps, a, p, stream, pdl)
                               : launch_x<LI_WTYPE_Q8_0, kTcSwiGLU>(maps, a, p, stream, pdl);
    case kTcConv: return q4 ? launch_x<LI_WTYPE_Q4_K, kTcConv>(maps, a, p, stream, pdl)
                             : launch_x<LI_WTYPE_Q8_0, kTcConv>(maps, a, p, stream, pdl);
    default: return LI_ERR_BAD_ARG;
    }
}
}  // namespace

int tc_gemm_launch(const TcArgs &a, cudaStream_t stream, bool pdl) {
    {
        TcxPlan px;
        if (planx(a, &px, false) == 0) {
            if (a.x_npad != px.Npad) return LI_ERR_BAD_ARG;   // X16 must be tiled for this kernel
            return launch_tcx(a, px, stream, pdl);
        }
    }
    TcPlan p;
    int rc = plan(a, &p);
    if (rc) return rc;
    if (a.x_npad != p.Npad) return LI_ERR_BAD_ARG;       // X16 must be tiled with the kernel's row padding
    const size_t rb = li_row_bytes(a.wtype, a.K);
    CUtensorMap maps[4];
    memset(maps, 0, sizeof(maps));
    const int nw = a.epi == kTcSwiGLU ? 2 : a.n_seg;
    for (int s = 0; s < 3; ++s) {
        const int src = s < nw ? s : 0;
        const int rows = a.epi == kTcSwiGLU ? a.seg_rows[0] : a.seg_rows[src];
        if (!aligned16(a.W[src])) return LI_ERR_MISALIGNED;
        rc = encode_2d(&maps[s], CU_TENSOR_MAP_DATA_TYPE_UINT32, a.W[src], rb / 4, (uint64_t)rows, rb,
                       (uint32_t)(p.RB / 4), kBM, CU_TENSOR_MAP_SWIZZLE_NONE);
        if (rc) return rc;
    }
    if (!aligned16(a.X16)) return LI_ERR_MISALIGNED;   // X slots come by bulk copies (no tensor map)
    const bool q4 = a.wtype == LI_WTYPE_Q4_K;
    switch (a.epi) {
    case kTcStore: return q4 ? launch_kernel<LI_WTYPE_Q4_K, kTcStore>(maps, a, p, stream, pdl)
                              : launch_kernel<LI_WTYPE_Q8_0, kTcStore>(maps, a, p, stream, pdl);
    case kTcSwiGLU:
        if (p.pair)
            return q4 ? launch_kernel<LI_WTYPE_Q4_K, kTcSwiGLUPair>(maps, a, p, stream, pdl)
                      : launch_kernel<LI_WTYPE_Q8_0, kTcSwiGLUPair>(maps, a, p, stream, pdl);
        return q4 ? launch_kernel<LI_WTYPE_Q4_K, kTcSwiGLU>(maps, a, p, stream, pdl)
                  : launch_kernel<LI_WTYPE_Q8_0, kTcSwiGLU>(maps, a, p, stream, pdl);
    case kTcConv: return q4 ? launch_kernel<LI_WTYPE_Q4_K, kTcConv>(maps, a, p, stream, pdl)
                             : launch_kernel<LI_WTYPE_Q8_0, kTcConv>(maps, a, p, stream, pdl);
    default: return LI_ERR_BAD_ARG;
    }
}

}  // namespace li
