// umma.cuh -- large per-expert groups on the 5th-generation tensor cores
// (tcgen05): fused dequantise + grouped GEMM with TMEM operands and
// accumulators.
//
// Where the decode kernels (gemv_stream.cuh) stream each expert's weights once
// per chunk of a few tokens, this kernel reads them once per block of up to
// 256 tokens of that expert.  One item = (expert, block of 128 output rows,
// block of n <= 256 tokens).  Per item the K range streams through three
// rings:
//   raw    quantised weight bytes of one super-block (256 columns) of the
//          item's 128 rows: one bulk copy per 8-row tile of the tiled layout
//          (gemv_stream.cuh), issued by the producer warp;
//   B      the tokens' activations, f16, 64 columns x n rows, one TMA tensor
//          load per 16 rows from the grouped activation matrix (rows in
//          dispatch order), 128-byte swizzled (the K-major canonical layout
//          of the MMA's shared-memory operand);
//   A      the dequantised weights, f16, 128 rows x 64 columns, written by the
//          dequantising warps straight into tensor memory (tcgen05.st), so
//          shared memory carries only the raw bytes and B.
// One thread issues tcgen05.mma (kind::f16, M = 128, N = n rounded up to 16,
// A from tensor memory, B from shared memory, f32 accumulators in tensor
// memory) four times per 64 columns and commits each A / B slot back to its
// ring.  Gate/up items hold 64 gate rows (accumulator lanes 0-63) and the same
// 64 up rows (lanes 64-127) so each B tile is read once for both; the
// epilogue pairs them through shared memory and applies SwiGLU, writing the
// down projection's f16 input.  Down items write f32 rows for the combine.
//
// Precision: weights dequantised to f16 (one rounding of a*q - b after the
// scales are rounded to f16), activations rounded to f16, products summed in
// f32.  Every wait is bounded (2 s or the CTA's abort flag); tensor memory is
// released on every exit path.  No clusters, no multicast.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>

#include "common.cuh"
#include "gemv.cuh"
#include "gemv_imma.cuh"
#include "gemv_stream.cuh"
#include "gemv_tma.cuh"
#include "umma_host.h"

namespace qrm {

// ------------------------------------------------------------ tcgen05 / TMA
__device__ __forceinline__ void tmem_alloc(uint32_t smem_dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_dst), "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// D[tmem] (+)= A[tmem] * B[smem]^T, kind::f16, one CTA
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// arrive on `bar` once every tcgen05.mma this thread issued so far has completed
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
        "%14, %15, %16};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&v)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
                 "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
                 : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}
// 2-D tensor tile load (no multicast) completing on `bar`
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// Shared-memory matrix descriptor of a K-major operand in the 128-byte
// swizzled canonical layout: rows of 128 bytes, 8-row groups 1024 bytes apart
// (stride byte offset), leading byte offset 16 (unused by this layout),
// descriptor version 1, swizzle mode 2 (128 B).  The operand must start on a
// 1024-byte boundary (base offset 0); the K slices of one 128-byte row are
// addressed by advancing the start address by 32 bytes per 16 f16 columns.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// Instruction descriptor of kind::f16: f32 accumulators, f16 A and B, both
// K-major, M = 128, N (multiple of 16, <= 256).
__host__ __device__ constexpr uint32_t umma_idesc_f16(int n) {
    return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

// ------------------------------------------------------------ geometry
constexpr int kUmmaRawRingMax = 6;    // raw stages (super-blocks) in flight, at most
constexpr int kUmmaBRingMax = 8;      // B tiles in flight, at most
constexpr int kUmmaARing = 4;         // A slots in tensor memory
// tokens per item: one tcgen05.mma (M = 128, K = 16) occupies the tensor pipe
// for about as long as N = 184 columns take, so N up to 192 keeps it busy; two
// 192-column accumulators and four 32-column A slots fill tensor memory
constexpr int kUmmaMaxN = 192;
constexpr int kUmmaBBytes = kUmmaMaxN * 128;
constexpr int kUmmaAccCols = kUmmaMaxN;   // one accumulator; two alternate between items
constexpr int kUmmaTmemCols = 512;    // accumulators [0, 384) + A slots [384, 512)
constexpr int kUmmaAColBase = 2 * kUmmaAccCols;
static_assert(kUmmaAColBase + 32 * kUmmaARing <= kUmmaTmemCols, "tensor memory columns");
constexpr int kUmmaWarps = 23;        // raw producer, MMA, 4 epilogue, 16 dequantising, B producer
constexpr int kUmmaEpiWarp0 = 2;
constexpr int kUmmaDqWarp0 = 6;
constexpr int kUmmaDqWarps = 16;      // 4 per tensor-memory lane quarter, 16 columns each
constexpr int kUmmaBWarp = 22;
constexpr int kUmmaStageBytes = 2 * 4096;   // epilogue exchange: 2 quarter pairs x 32 rows x 32 columns x 4 B

// bytes of one raw stage: 16 tile chunks of one super-block, each padded by 16
// bytes so that the four tiles a warp reads start on different banks
__host__ __device__ inline int umma_chunk_pitch(int fmt) { return tile_chunk_bytes(fmt) + 16; }
__host__ __device__ inline int umma_raw_bytes(int fmt) { return 16 * umma_chunk_pitch(fmt); }


struct UmmaParams {
    const MatDev* mats;        // [E+1][3]
    const UmmaItem* items;
    const int32_t* n_items;
    int K;                     // columns of the matrices (d for gate/up, f for down)
    int rows;                  // rows of one matrix (f for gate/up, d for down)
    int shared_pos;            // activation rows >= shared_pos belong to the shared expert
    float limit;               // SwiGLU limit (gate/up)
    __half* h_out;             // gate/up: [rows_total][f] f16 (the down input)
    float* y_routed;           // down: [T*k][d]
    float* y_shared;           // down: [T][d]
    int32_t* err;
};

// ------------------------------------------------------------ dequantisation
// Row r of the item (0..127) in a raw stage: tile chunk r / 8, row r % 8.
// `part` selects columns [16 part, 16 part + 16) of sub-step j (64 columns)
// of the super-block; the 16 weights come out as 8 f16 pairs (word c = weights
// 2c, 2c+1 of the part).

__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 bits_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// w = (code - off) * a + nb for the 8 codes (bytes) of two words -> 4 pairs;
// the codes enter as the f16 values 1024 + code (exact), so code - off is exact
__device__ __forceinline__ void dq_words(uint32_t c0, uint32_t c1, __half2 off, __half2 a, __half2 nb, uint32_t* out) {
    const uint32_t p[4] = {prmt(c0, 0x64646464u, 0x4140u), prmt(c0, 0x64646464u, 0x4342u),
                           prmt(c1, 0x64646464u, 0x4140u), prmt(c1, 0x64646464u, 0x4342u)};
#pragma unroll
    for (int i = 0; i < 4; i++) out[i] = h2_bits(__hfma2(__hsub2(bits_h2(p[i]), off), a, nb));
}

// The row's per-super-block header, read once per raw stage: Q4_K d, dmin
// and scales; Q8_0 / Q4_0 the eight blocks' d; Q6_K the 16 scales (h) and d
// (e); TRI the four blocks' scales (h.x, h.y).
struct UmmaHdr {
    uint4 h;
    uint32_t e;
};
template <int FMT>
__device__ __forceinline__ UmmaHdr umma_row_header(const uint8_t* raw, int r) {
    const uint8_t* chunk = raw + (r >> 3) * umma_chunk_pitch(FMT);
    const int rr = r & 7;
    UmmaHdr hd;
    hd.e = 0;
    if (FMT == Q6_K) {
        hd.h = *reinterpret_cast<const uint4*>(chunk + 1536 + 16 * rr);
        hd.e = *reinterpret_cast<const uint16_t*>(chunk + 1664 + 2 * rr);
    } else if (FMT == TRI) {
        const uint2 v = *reinterpret_cast<const uint2*>(chunk + 512 + 8 * rr);
        hd.h = make_uint4(v.x, v.y, 0u, 0u);
    } else {
        hd.h = *reinterpret_cast<const uint4*>(chunk + 16 * rr);
    }
    return hd;
}

// f16 pairs (t(c0), t(c1)) of the TRI codes in a nibble (c0 = low two bits):
// code 01 -> +1, 10 -> -1, 00 and 11 -> 0 (BlockDequantizer.cs:258-276)
__device__ __forceinline__ uint32_t tri_pair_bits(int n) {
    const int c0 = n & 3, c1 = n >> 2;
    const float t0 = c0 == 1 ? 1.f : c0 == 2 ? -1.f : 0.f, t1 = c1 == 1 ? 1.f : c1 == 2 ? -1.f : 0.f;
    return h2_bits(__floats2half2_rn(t0, t1));
}

template <int FMT>
__device__ __forceinline__ void umma_dequant(const uint8_t* raw, const UmmaHdr& hd, const uint32_t* tri_lut, int r,
                                             int j, int part, uint32_t (&w)[8]) {
    const uint8_t* chunk = raw + (r >> 3) * umma_chunk_pitch(FMT);
    const int rr = r & 7, half = part >> 1, sub = part & 1;
    const uint4& h4 = hd.h;
    if (FMT == TRI) {
        // codes[r][blk][16]: weight i of block j at byte i/4, bits 2(i & 3); part p
        // = weights 16p..16p+15 = one word; w = s * t exactly (s is f16)
        const uint32_t x = *reinterpret_cast<const uint32_t*>(chunk + 64 * rr + 16 * j + 4 * part);
        const uint32_t sw = j < 2 ? h4.x : h4.y;
        const __half2 s2 = __half2half2(__ushort_as_half((uint16_t)(sw >> (16 * (j & 1)))));
#pragma unroll
        for (int k = 0; k < 8; k++) w[k] = h2_bits(__hmul2(bits_h2(tri_lut[(x >> (4 * k)) & 15u]), s2));
    } else if (FMT == Q6_K) {
        // DequantQ6_K (BlockDequantizer.cs:228-256): half h = j / 2 of the block
        // (128 weights); in it, group g of 32 (q1..q4) takes ql[64h + 32(g & 1) + l]
        // (low nibble for g < 2, high for g >= 2) and bits 2g of qh[32h + l],
        // scale sc[8h + l/16 + 2g]; w = d * sc * (q - 32)
        const int hh = j >> 1, local = 64 * (j & 1) + 16 * part, g = local >> 5, l0 = local & 31;
        const uint4 ql = *reinterpret_cast<const uint4*>(chunk + 128 * rr + 64 * hh + 32 * (g & 1) + l0);
        const uint4 qh = *reinterpret_cast<const uint4*>(chunk + 1024 + 64 * rr + 32 * hh + l0);
        const int si = 8 * hh + (l0 >> 4) + 2 * g;
        const uint32_t scw = si < 4 ? h4.x : si < 8 ? h4.y : si < 12 ? h4.z : h4.w;
        const int sc = (int)(int8_t)((scw >> (8 * (si & 3))) & 0xFF);
        const float d = h2f((uint16_t)hd.e);
        const __half2 a = __float2half2_rn(d * (float)sc);
        const __half2 nb = __float2half2_rn(0.f);
        const __half2 off = __float2half2_rn(1056.f);   // 1024 + 32
        const int ls = 4 * (g >> 1), hs = 2 * g;
        const uint32_t lw[4] = {ql.x, ql.y, ql.z, ql.w}, hw[4] = {qh.x, qh.y, qh.z, qh.w};
        uint32_t qq[4];
#pragma unroll
        for (int i = 0; i < 4; i++) qq[i] = ((lw[i] >> ls) & 0x0F0F0F0Fu) | (((hw[i] >> hs) & 0x03030303u) << 4);
        dq_words(qq[0], qq[1], off, a, nb, &w[0]);
        dq_words(qq[2], qq[3], off, a, nb, &w[4]);
    } else if (FMT == Q4_K) {
        // hdr[8][16] | qs[4 pairs][8 rows][32]: in pair j, byte i holds weight i
        // of sub-block 2j (low nibble) and of sub-block 2j+1 (high nibble)
        const uint4 q4 = *reinterpret_cast<const uint4*>(chunk + 128 + 256 * j + 32 * rr + 16 * sub);
        const int sb = 2 * j + half;
        // GetScaleMinK4 (BlockDequantizer.cs:155-166) on scale bytes q[0..11]
        // (header words y, z, w)
        const int bsel = 8 * (sb & 3);
        const uint32_t b0 = (h4.y >> bsel) & 0xFF, b4 = (h4.z >> bsel) & 0xFF, b8 = (h4.w >> bsel) & 0xFF;
        int sc, mn;
        if (sb < 4) {
            sc = b0 & 63;                            // q[sb]
            mn = b4 & 63;                            // q[sb + 4]
        } else {
            sc = (b8 & 0xF) | ((b0 >> 6) << 4);      // q[sb + 4], q[sb - 4]
            mn = (b8 >> 4) | ((b4 >> 6) << 4);       // q[sb + 4], q[sb]
        }
        const float d = h2f((uint16_t)(h4.x & 0xFFFF)), dmin = h2f((uint16_t)(h4.x >> 16));
        // w = a*q - b in f32, one rounding to f16: b is about the size of the
        // largest a*q, so rounding a or b to f16 first would leave an error
        // shared by all 32 weights of the sub-block.  The code enters as the
        // float 0.5 + q/256 (byte placed in mantissa bits 16-19 of 2^-1), so one
        // FMA gives (0.5 + q/256)*256a + (nb - 128a) = a*q + nb; the constant's
        // f32 rounding (~1e-7 of a weight) is far below the f16 rounding
        const float a = d * (float)sc, nb = -(dmin * (float)mn);
        const float2 a2 = make_float2(256.f * a, 256.f * a);
        const float c = nb - 128.f * a;
        const float2 c2 = make_float2(c, c);
        const uint32_t qs[4] = {q4.x, q4.y, q4.z, q4.w};
        const int sh = 4 * half;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const uint32_t x = (qs[i] >> sh) & 0x0F0F0F0Fu;
#pragma unroll
            for (int pr = 0; pr < 2; pr++) {
                const float2 m = make_float2(__uint_as_float(prmt(x, 0x3F000000u, 0x7054u | ((2u * pr) << 8))),
                                             __uint_as_float(prmt(x, 0x3F000000u, 0x7054u | ((2u * pr + 1) << 8))));
                const float2 w2 = ffma2(m, a2, c2);
                w[2 * i + pr] = h2_bits(__floats2half2_rn(w2.x, w2.y));
            }
        }
    } else if (FMT == Q8_0) {
        // d[8 rows][8 blocks][2] | qs[8 blocks][8 rows][32] (int8); w = d * q, one rounding
        const int blk = 2 * j + half;
        const uint32_t dw = blk < 2 ? h4.x : blk < 4 ? h4.y : blk < 6 ? h4.z : h4.w;
        const float d = h2f((uint16_t)(dw >> (16 * (blk & 1))));
        const uint4 q4 = *reinterpret_cast<const uint4*>(chunk + 128 + 256 * blk + 32 * rr + 16 * sub);
        const __half2 a = __float2half2_rn(d);
        const __half2 nb = __float2half2_rn(0.f);
        const __half2 off = __float2half2_rn(1152.f);   // 1024 + 128 (codes biased by 128)
        dq_words(q4.x ^ 0x80808080u, q4.y ^ 0x80808080u, off, a, nb, &w[0]);
        dq_words(q4.z ^ 0x80808080u, q4.w ^ 0x80808080u, off, a, nb, &w[4]);
    } else {  // Q4_0: d[8][8][2] | pad[8][8][2] | qs[8 blocks][8 rows][16]; low nibbles = weights 0-15
        const int blk = 2 * j + half;
        const uint32_t dw = blk < 2 ? h4.x : blk < 4 ? h4.y : blk < 6 ? h4.z : h4.w;
        const float d = h2f((uint16_t)(dw >> (16 * (blk & 1))));
        const uint4 q4 = *reinterpret_cast<const uint4*>(chunk + 256 + 128 * blk + 16 * rr);
        const __half2 a = __float2half2_rn(d);
        const __half2 nb = __float2half2_rn(0.f);
        const __half2 off = __float2half2_rn(1032.f);   // 1024 + 8
        const int sh = 4 * sub;
        dq_words((q4.x >> sh) & 0x0F0F0F0Fu, (q4.y >> sh) & 0x0F0F0F0Fu, off, a, nb, &w[0]);
        dq_words((q4.z >> sh) & 0x0F0F0F0Fu, (q4.w >> sh) & 0x0F0F0F0Fu, off, a, nb, &w[4]);
    }
}

// SiLU(g) * u (Glm5Ops.LimitedSwiglu clamps first when limit > 0) with the
// fast exponential: the expert products of this path carry f16 operands, so
// the last bits of the reference's MathF.Exp do not reach the 1e-3 bound
__device__ __forceinline__ float swiglu_fast(float g, float u, float limit) {
    if (limit > 0.f) {
        g = fminf(g, limit);
        u = fminf(fmaxf(u, -limit), limit);
    }
    return __fdividef(g, 1.f + __expf(-g)) * u;
}

// ------------------------------------------------------------ kernel
// Shared memory: [control 1 KB][raw ring][B ring (1024-aligned)][epilogue exchange]
struct UmmaSmem {
    int raw_stages;     // raw ring depth
    int raw_bytes;      // bytes of one raw stage
    int b_stages;       // B ring depth
    size_t b_off, x_off, total;
};
// Ring depths: at least three raw stages (two for the largest formats), as
// many B tiles as fit up to 8, then more raw stages with what is left (two
// raw stages and five B tiles for the Q8_0 shared expert of C5 measured the
// same at T 4096, and slower for C4).
__host__ inline UmmaSmem umma_smem(int fa, int fb) {
    UmmaSmem s;
    s.raw_bytes = std::max(umma_raw_bytes(fa), umma_raw_bytes(fb));
    const int budget = 227 * 1024 - 1024 /* alignment slack */ - 1024 /* control */ - 1024 /* B alignment */ -
                       kUmmaStageBytes;
    const int raw_min = 3 * s.raw_bytes + 4 * kUmmaBBytes <= budget ? 3 : 2;
    s.b_stages = std::min(kUmmaBRingMax, (budget - raw_min * s.raw_bytes) / kUmmaBBytes);
    s.raw_stages = std::min(kUmmaRawRingMax, (budget - s.b_stages * kUmmaBBytes) / s.raw_bytes);
    s.b_off = ((size_t)1024 + (size_t)s.raw_stages * s.raw_bytes + 1023) / 1024 * 1024;
    s.x_off = s.b_off + (size_t)s.b_stages * kUmmaBBytes;
    s.total = s.x_off + kUmmaStageBytes + 1024;
    return s;
}

// FA: format of the routed experts, FB: of the shared expert (items whose
// activation rows start at or after p.shared_pos)
template <int FA, int FB, bool GATEUP>
__global__ void __launch_bounds__(kUmmaWarps * 32, 1)
expert_umma_kernel(const __grid_constant__ CUtensorMap act_map, UmmaParams p, int raw_stages, int raw_bytes,
                   int b_stages, int b_off, int x_off) {
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte aligned base (the swizzled B tiles need it)
    uint8_t* sm = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    uint64_t* raw_full = reinterpret_cast<uint64_t*>(sm);
    uint64_t* raw_empty = raw_full + kUmmaRawRingMax;
    uint64_t* b_full = raw_empty + kUmmaRawRingMax;
    uint64_t* b_empty = b_full + kUmmaBRingMax;
    uint64_t* a_full = b_empty + kUmmaBRingMax;
    uint64_t* a_empty = a_full + kUmmaARing;
    uint64_t* acc_full = a_empty + kUmmaARing;     // [2]
    uint64_t* acc_empty = acc_full + 2;            // [2]
    uint64_t* done_bar = acc_empty + 2;
    uint64_t* x_full = done_bar + 1;    // [2] epilogue exchange per quarter pair
    uint64_t* x_empty = x_full + 2;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + 512);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + 520);
    uint32_t* tri_lut = reinterpret_cast<uint32_t*>(sm + 576);   // [16] TRI nibble -> f16 pair
    uint8_t* raw = sm + 1024;
    uint8_t* bring = sm + b_off;
    float* xch = reinterpret_cast<float*>(sm + x_off);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int RS = raw_stages, BS = b_stages;
    if (tid == 0) {
        for (int i = 0; i < RS; i++) {
            mbar_init(&raw_full[i], 1);
            mbar_init(&raw_empty[i], kUmmaDqWarps);
        }
        for (int i = 0; i < BS; i++) {
            mbar_init(&b_full[i], 1);
            mbar_init(&b_empty[i], 1);
        }
        for (int i = 0; i < kUmmaARing; i++) {
            mbar_init(&a_full[i], kUmmaDqWarps);
            mbar_init(&a_empty[i], 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], 4);
        }
        mbar_init(done_bar, 1);
        for (int i = 0; i < 2; i++) {
            mbar_init(&x_full[i], 1);
            mbar_init(&x_empty[i], 1);
        }
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (tid < 16) {
        tri_lut[tid] = tri_pair_bits(tid);
    }
    if (warp == 1) tmem_alloc(smem_u32(tmem_slot), kUmmaTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int n_items = *p.n_items;
    const int K = p.K, nsb = K / 256, nsub = K / 64;

    if (warp == 0) {
        // ------------------------------------------------ raw producer: weight bytes
        bool ok = true;
        uint32_t gr = 0;   // raw stages issued
        for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
            const UmmaItem item = p.items[it];
            const MatDev* md = p.mats + item.mat;
            const bool shi = item.pos >= p.shared_pos;
            const int cb = shi ? tile_chunk_bytes(FB) : tile_chunk_bytes(FA);
            for (int sb = 0; sb < nsb; sb++) {
                // raw stage: 16 tile chunks of super-block sb
                const int s = gr % RS;
                if (gr >= (uint32_t)RS) {
                    const bool w = lane == 0 ? mbar_wait_abort(&raw_empty[s], ((gr / RS) & 1u) ^ 1u, abort_flag) : true;
                    if (!__shfl_sync(0xffffffffu, (int)w, 0)) { ok = false; break; }
                }
                if (lane == 0) mbar_arrive_expect_tx(&raw_full[s], (uint32_t)(16 * cb));
                __syncwarp();
                if (lane < 16) {
                    int tile;
                    const MatDev* m;
                    if (GATEUP) { m = md + (lane >> 3); tile = item.rb * 8 + (lane & 7); }
                    else { m = md; tile = item.rb * 16 + lane; }
                    bulk_g2s(raw + (size_t)s * raw_bytes + lane * (cb + 16), m->base + ((long long)tile * nsb + sb) * cb,
                             (uint32_t)cb, &raw_full[s]);
                }
                gr++;
            }
        }
        if (!ok && lane == 0) {
            *abort_flag = 1;
            atomicOr(p.err, (int)ERR_TIMEOUT);
            // copies already issued must land before the CTA exits
            for (uint32_t i = gr > (uint32_t)RS ? gr - RS : 0; i < gr; i++) mbar_wait(&raw_full[i % RS], (i / RS) & 1u);
        }
    } else if (warp == kUmmaBWarp) {
        // ------------------------------------------------ B producer: activation tiles
        bool ok = true;
        uint32_t gb = 0;   // B tiles issued
        for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
            const UmmaItem item = p.items[it];
            const int nt16 = (item.n + 15) >> 4;
            for (int ks = 0; ks < nsub; ks++) {
                const int s = gb % BS;
                if (gb >= (uint32_t)BS) {
                    const bool w = lane == 0 ? mbar_wait_abort(&b_empty[s], ((gb / BS) & 1u) ^ 1u, abort_flag) : true;
                    if (!__shfl_sync(0xffffffffu, (int)w, 0)) { ok = false; break; }
                }
                if (lane == 0) mbar_arrive_expect_tx(&b_full[s], (uint32_t)(nt16 * 2048));
                __syncwarp();
                if (lane < nt16)
                    tma_load_2d(bring + (size_t)s * kUmmaBBytes + lane * 2048, &act_map, ks * 64, item.pos + 16 * lane,
                                &b_full[s]);
                gb++;
            }
        }
        if (!ok && lane == 0) {
            *abort_flag = 1;
            atomicOr(p.err, (int)ERR_TIMEOUT);
            for (uint32_t i = gb > (uint32_t)BS ? gb - BS : 0; i < gb; i++) mbar_wait(&b_full[i % BS], (i / BS) & 1u);
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer (one thread)
        if (lane == 0) {
            bool ok = true;
            uint32_t ga = 0, gb = 0, gi = 0;
            for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x, gi++) {
                const UmmaItem item = p.items[it];
                const int n16 = (item.n + 15) & ~15;
                const uint32_t idesc = umma_idesc_f16(n16);
                // accumulators alternate between items: the epilogue of one item
                // overlaps the MMAs of the next
                const uint32_t ab = gi & 1u, acc = tmem + kUmmaAccCols * ab;
                if (gi >= 2) {
                    if (!mbar_wait_abort(&acc_empty[ab], ((gi >> 1) - 1) & 1u, abort_flag)) { ok = false; break; }
                    tc_fence_after();
                }
                for (int ks = 0; ks < nsub; ks++) {
                    const int as = ga % kUmmaARing, bs = gb % BS;
                    if (!mbar_wait_abort(&a_full[as], (ga / kUmmaARing) & 1u, abort_flag) ||
                        !mbar_wait_abort(&b_full[bs], (gb / BS) & 1u, abort_flag)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t a_t = tmem + kUmmaAColBase + 32 * as;
                    const uint32_t b_s = smem_u32(bring + (size_t)bs * kUmmaBBytes);
#pragma unroll
                    for (int kk = 0; kk < 4; kk++)
                        umma_ts(acc, a_t + 8 * kk, sw128_desc(b_s + 32 * kk), idesc, (ks | kk) ? 1u : 0u);
                    umma_commit(&a_empty[as]);
                    umma_commit(&b_empty[bs]);
                    ga++;
                    gb++;
                }
                if (ok) umma_commit(&acc_full[ab]);
            }
            if (!ok) {
                *abort_flag = 1;
                atomicOr(p.err, (int)ERR_TIMEOUT);
            }
            // every MMA of this CTA has completed before tensor memory is released
            umma_commit(done_bar);
            mbar_wait(done_bar, 0u);
        }
        __syncwarp();
    } else if (warp < kUmmaDqWarp0) {
        // ------------------------------------------------ epilogue (lane quarter warp % 4)
        const int q = warp & 3;
        const uint32_t lane_base = (uint32_t)(32 * q) << 16;
        uint32_t gi = 0, gx = 0;   // items, exchange rounds of this warp's pair
        for (int it = blockIdx.x; it < n_items; it += gridDim.x, gi++) {
            const UmmaItem item = p.items[it];
            const uint32_t ab = gi & 1u, acc = tmem + kUmmaAccCols * ab;
            if (!warp_wait(&acc_full[ab], (gi >> 1) & 1u, abort_flag, p.err)) break;
            tc_fence_after();
            if (GATEUP) {
                // lanes 0-63 gate rows, 64-127 up rows: quarters 2, 3 hand their up
                // values to quarters 0, 1 through shared memory, 32 columns at a
                // time (bounded mbarrier hand-offs: a warp that gives up cannot
                // leave its partner waiting)
                const int pair = q & 1;
                float* xp = xch + pair * 1024;
                const int f = p.rows;
                const int row = item.rb * 64 + 32 * pair + lane;
                bool ok = true;
                for (int c0 = 0; c0 < item.n && ok; c0 += 32, gx++) {
                    float v[2][16];
                    tmem_ld16(acc + lane_base + c0, v[0]);
                    tmem_ld16(acc + lane_base + c0 + 16, v[1]);
                    if (q >= 2) {
                        if (gx > 0 && !warp_wait(&x_empty[pair], (gx - 1) & 1u, abort_flag, p.err)) { ok = false; break; }
#pragma unroll
                        for (int c = 0; c < 32; c++) xp[c * 32 + lane] = v[c >> 4][c & 15];
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&x_full[pair]);
                    } else {
                        if (!warp_wait(&x_full[pair], gx & 1u, abort_flag, p.err)) { ok = false; break; }
                        const int nc = min(32, item.n - c0);
                        __half* hp = p.h_out + (size_t)(item.pos + c0) * f + row;
#pragma unroll
                        for (int c = 0; c < 32; c++) {
                            if (c < nc) {
                                const float g = v[c >> 4][c & 15];
                                const float u = xp[c * 32 + lane];
                                hp[(size_t)c * f] = __float2half_rn(swiglu_fast(g, u, p.limit));
                            }
                        }
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&x_empty[pair]);
                    }
                }
                if (!ok) break;
            } else {
                const int row = item.rb * 128 + 32 * q + lane;
                const int d = p.rows;
                for (int c0 = 0; c0 < item.n; c0 += 16) {
                    float v[16];
                    tmem_ld16(acc + lane_base + c0, v);
                    const int nc = min(16, item.n - c0);
#pragma unroll
                    for (int c = 0; c < 16; c++) {
                        if (c < nc) {
                            const int pos = item.pos + c0 + c;
                            float* dst = pos >= p.shared_pos ? p.y_shared + (size_t)(pos - p.shared_pos) * d
                                                             : p.y_routed + (size_t)pos * d;
                            dst[row] = v[c];
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[ab]);
        }
    } else {
        // ------------------------------------------------ dequantising warps
        const int dw = warp - kUmmaDqWarp0;
        const int q = warp & 3, part = dw >> 2;
        const int r = 32 * q + lane;   // row of the item (tensor-memory lane)
        const uint32_t lane_base = (uint32_t)(32 * q) << 16;
        const uint32_t a_base = tmem + lane_base + kUmmaAColBase + 8 * part;
        bool ok = true;
        uint32_t gr = 0, ga = 0;       // raw stages consumed, A slots stored
        bool pend = false;             // stores of slots ga-2, ga-1 in flight
        // two sub-steps per round; the stores of one round complete while the
        // next round is computed
        for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
            const bool shi = p.items[it].pos >= p.shared_pos;
            for (int sb = 0; sb < nsb && ok; sb++) {
                const int s = gr % RS;
                if (!warp_wait(&raw_full[s], (gr / RS) & 1u, abort_flag, p.err)) { ok = false; break; }
                const uint8_t* st = raw + (size_t)s * raw_bytes;
                const UmmaHdr hdr = shi ? umma_row_header<FB>(st, r) : umma_row_header<FA>(st, r);
                for (int jp = 0; jp < 2; jp++) {
                    uint32_t w0[8], w1[8];
                    if (shi) {
                        umma_dequant<FB>(st, hdr, tri_lut, r, 2 * jp, part, w0);
                        umma_dequant<FB>(st, hdr, tri_lut, r, 2 * jp + 1, part, w1);
                    } else {
                        umma_dequant<FA>(st, hdr, tri_lut, r, 2 * jp, part, w0);
                        umma_dequant<FA>(st, hdr, tri_lut, r, 2 * jp + 1, part, w1);
                    }
                    if (jp == 1) {
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&raw_empty[s]);   // the stage's bytes are in registers
                    }
                    if (pend) {
                        tmem_st_wait();
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) {
                            mbar_arrive(&a_full[(ga - 2) % kUmmaARing]);
                            mbar_arrive(&a_full[(ga - 1) % kUmmaARing]);
                        }
                        pend = false;
                    }
                    const int as0 = ga % kUmmaARing, as1 = (ga + 1) % kUmmaARing;
                    if (ga >= (uint32_t)kUmmaARing &&
                        (!warp_wait(&a_empty[as0], ((ga / kUmmaARing) & 1u) ^ 1u, abort_flag, p.err) ||
                         !warp_wait(&a_empty[as1], (((ga + 1) / kUmmaARing) & 1u) ^ 1u, abort_flag, p.err))) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    tmem_st8(a_base + 32 * as0, w0);
                    tmem_st8(a_base + 32 * as1, w1);
                    ga += 2;
                    pend = true;
                }
                gr++;
            }
        }
        // the last round's stores (also on the way out after a failed wait:
        // tensor memory is released only once they have completed)
        tmem_st_wait();
        if (pend && ok) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&a_full[(ga - 2) % kUmmaARing]);
                mbar_arrive(&a_full[(ga - 1) % kUmmaARing]);
            }
        }
    }
    // ---------------- teardown: every role is done (or gave up); free tensor memory
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, kUmmaTmemCols);
}

// ------------------------------------------------------------ helpers
// f16 activation rows in dispatch order: row pos < T*k is token perm[pos] / k,
// rows T*k + t (shared expert) are token t.
__global__ void umma_gather_kernel(const float* __restrict__ xn, const float* __restrict__ xn_shared,
                                   const int32_t* __restrict__ pos_tok, int Tk, int shared_rows, int d,
                                   __half* __restrict__ out) {
    const int rows = Tk + shared_rows;
    const int v8 = d / 8;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < (long long)rows * v8;
         i += (long long)gridDim.x * blockDim.x) {
        const int row = (int)(i / v8), c = (int)(i - (long long)row * v8);
        const float* src = row < Tk ? xn + (size_t)pos_tok[row] * d : xn_shared + (size_t)(row - Tk) * d;
        const float4 a = __ldg(reinterpret_cast<const float4*>(src) + 2 * c);
        const float4 b = __ldg(reinterpret_cast<const float4*>(src) + 2 * c + 1);
        uint4 o;
        o.x = h2_bits(__floats2half2_rn(a.x, a.y));
        o.y = h2_bits(__floats2half2_rn(a.z, a.w));
        o.z = h2_bits(__floats2half2_rn(b.x, b.y));
        o.w = h2_bits(__floats2half2_rn(b.z, b.w));
        reinterpret_cast<uint4*>(out + (size_t)row * d)[c] = o;
    }
}

// Items of both expert stages from the dispatch's slot table (one warp):
// per routed slot (and the shared expert) its tokens in blocks of <= 256
// (balanced, multiples of 16 where possible) times the row blocks.
__global__ void umma_plan_kernel(const int4* __restrict__ slot_info, const int32_t* __restrict__ n_active,
                                 int has_shared, int Tk, int rb_gateup, int rb_down, int E, UmmaItem* gu_items,
                                 int32_t* gu_count, UmmaItem* dn_items, int32_t* dn_count, int cap) {
    const int na = *n_active;
    const int nslots = na + (has_shared ? 1 : 0);
    int ngu = 0, ndn = 0;
    for (int s = 0; s < nslots; s++) {
        const int4 si = slot_info[s];   // expert, first position, tokens, first token
        const bool sh = s == na;
        const int e = sh ? E : si.x, pos0 = sh ? Tk : si.y, n = si.z;
        if (n <= 0) continue;
        const int nb = (n + kUmmaMaxN - 1) / kUmmaMaxN;
        const int per = ((n + nb - 1) / nb + 15) & ~15;
        for (int b = 0; b * per < n; b++) {
            const int pos = pos0 + b * per, cnt = min(per, n - b * per);
            for (int rb = threadIdx.x; rb < rb_gateup; rb += 32)
                if (ngu + rb < cap) gu_items[ngu + rb] = UmmaItem{e * 3 + 0, rb, pos, cnt};
            for (int rb = threadIdx.x; rb < rb_down; rb += 32)
                if (ndn + rb < cap) dn_items[ndn + rb] = UmmaItem{e * 3 + 2, rb, pos, cnt};
            ngu += rb_gateup;
            ndn += rb_down;
        }
    }
    if (threadIdx.x == 0) {
        *gu_count = min(ngu, cap);
        *dn_count = min(ndn, cap);
    }
}

}  // namespace qrm
