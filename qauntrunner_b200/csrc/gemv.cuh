// gemv.cuh -- fused dequantise + dot products of the expert matrices.
//
// The reference runs every expert product as DotKernels.MatVecParallel over
// the compressed rows (DotKernels.cs:610-629 -> DotQ4_0 132-179, DotQ8_0
// 184-205, DotQ4_K 325-357, DotQ6_K 423-451, DotTri 456-471), one token and
// one expert at a time.  Here one persistent kernel walks a work list of
// (expert, row tile) items for all experts the batch selected (plus the GLM
// shared expert) and computes the rows of the tile for every token routed to
// that expert, so each weight byte leaves HBM once per forward.
//
// Thread layout: a CTA has one thread per 32-weight "unit" of a row
// (cols/32 units, rounded up to whole warps).  Each thread keeps its unit's
// activations in registers, loads its unit of every row of the tile with
// aligned vector loads (16/8-byte loads; the formats whose blocks are not
// 16-byte multiples are stored field-split, see MatDev), accumulates in f32,
// and the CTA reduces the row sums with a transposing warp reduction plus one
// shared-memory pass -- a fixed order, so results are deterministic.
//
// Integer codes become floats without a conversion instruction: a code byte b
// placed in the mantissa of 2.0f (bits 16..22 for b < 128, 15..22 otherwise)
// reads as F = 2 + b/64 (or 2 + b/128), so sum(b*x) = 64*(sum(F*x) - 2*sum(x))
// (or 128*(...)).  The cancellation costs at most ~5 of the 24 significand bits.
#pragma once
#include "common.cuh"
#include "glibc_expf.cuh"

namespace qrm {

__device__ __forceinline__ uint4 ld_stream16(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}
__device__ __forceinline__ uint2 ld_stream8(const void* p) {
    uint2 r;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];\n" : "=r"(r.x), "=r"(r.y) : "l"(p));
    return r;
}
__device__ __forceinline__ uint16_t ld_u16(const void* p) { return __ldg((const unsigned short*)p); }

// Byte K of w placed at bit POS of 0x40000000 reads as F = 2 + b * 2^(POS-22):
// POS 16 gives 2 + b/64 for b < 128 (bit 23 is the exponent's low bit, so
// larger bytes must use POS 15: 2 + b/128).  Written as shift and mask; the
// __byte_perm intrinsic made ptxas spill these kernels heavily.
template <int K, int POS>
__device__ __forceinline__ float bfk(uint32_t w) {
    uint32_t v = (8 * K <= POS) ? (w << (POS - 8 * K)) : (w >> (8 * K - POS));
    return __uint_as_float((v & (0xFFu << POS)) | 0x40000000u);
}

// sum_{k<4} F(byte k of w) * x[o+k]  (x passed by value so it stays in registers)
#define QRM_DOT4(w, X, o, acc, POS)                               \
    do {                                                          \
        (acc) = fmaf(bfk<0, POS>(w), (X)[(o) + 0], (acc));        \
        (acc) = fmaf(bfk<1, POS>(w), (X)[(o) + 1], (acc));        \
        (acc) = fmaf(bfk<2, POS>(w), (X)[(o) + 2], (acc));        \
        (acc) = fmaf(bfk<3, POS>(w), (X)[(o) + 3], (acc));        \
    } while (0)

// ---------------------------------------------------------------- units

// x column of register i (0..31) of unit u
template <int FMT>
__device__ __forceinline__ int unit_col(int u, int i);
template <> __device__ __forceinline__ int unit_col<Q4_K>(int u, int i) {
    int b = u >> 3, j = u & 7;
    return 256 * b + 64 * (j >> 1) + 16 * (j & 1) + (i & 15) + (i >> 4) * 32;
}
template <> __device__ __forceinline__ int unit_col<Q6_K>(int u, int i) {
    int b = u >> 3, uu = u & 7;
    return 256 * b + 128 * (uu >> 2) + 32 * (i >> 3) + 8 * (uu & 3) + (i & 7);
}
template <> __device__ __forceinline__ int unit_col<Q4_0>(int u, int i) { return 32 * u + i; }
template <> __device__ __forceinline__ int unit_col<Q8_0>(int u, int i) { return 32 * u + i; }
template <> __device__ __forceinline__ int unit_col<TRI>(int u, int i) { return 32 * u + i; }
// the raw formats: unit u = weights [32u, 32u + 32) of the row (256-weight
// blocks: block u / 8, quarter-pair u % 8)
template <> __device__ __forceinline__ int unit_col<Q2_K>(int u, int i) { return 32 * u + i; }
template <> __device__ __forceinline__ int unit_col<Q3_K>(int u, int i) { return 32 * u + i; }
template <> __device__ __forceinline__ int unit_col<Q5_K>(int u, int i) { return 32 * u + i; }
template <> __device__ __forceinline__ int unit_col<I8_BLK>(int u, int i) { return 32 * u + i; }
template <> __device__ __forceinline__ int unit_col<B1>(int u, int i) { return 32 * u + i; }
template <> __device__ __forceinline__ int unit_col<B1X>(int u, int i) { return 32 * u + i; }
template <> __device__ __forceinline__ int unit_col<T1E>(int u, int i) { return 32 * u + i; }
template <> __device__ __forceinline__ int unit_col<T1E_LO>(int u, int i) { return 32 * u + i; }

// Per-token activation registers of one unit and the partial sums the
// formats need.
struct XUnit {
    float x[32];
    float s[4];   // sums of x[0..8), [8..16), [16..24), [24..32)
};

template <int FMT>
__device__ __forceinline__ void load_x(XUnit& xu, const float* __restrict__ row, int u) {
#pragma unroll
    for (int q = 0; q < 8; q++) {
        int c = unit_col<FMT>(u, 4 * q);
        float4 v = __ldg((const float4*)(row + c));
        xu.x[4 * q] = v.x; xu.x[4 * q + 1] = v.y; xu.x[4 * q + 2] = v.z; xu.x[4 * q + 3] = v.w;
    }
#pragma unroll
    for (int g = 0; g < 4; g++) {
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < 8; i++) s += xu.x[8 * g + i];
        xu.s[g] = s;
    }
}

template <int FMT> struct WUnit;

// Q4_K: 144-byte blocks as in .qw; unit j = qs bytes [16j, 16j+16).
template <> struct WUnit<Q4_K> {
    uint4 hdr, qs;
    int j;
    __device__ __forceinline__ void load(const MatDev& m, int row, int u) {
        int bpr = m.cols >> 8;
        const uint8_t* blk = m.base + ((size_t)row * bpr + (u >> 3)) * 144;
        j = u & 7;
        hdr = __ldg((const uint4*)blk);
        qs = ld_stream16(blk + 16 + 16 * j);
    }
    __device__ __forceinline__ float dot(const XUnit& xu) const {
        // GetScaleMinK4 (BlockDequantizer.cs:155-166) for sub-blocks 2g, 2g+1
        const uint32_t s0 = hdr.y, s1 = hdr.z, s2 = hdr.w;  // scales[0..12)
        auto byte = [&](int i) -> uint32_t {
            uint32_t w = i < 4 ? s0 : (i < 8 ? s1 : s2);
            return (w >> (8 * (i & 3))) & 0xFF;
        };
        int g = j >> 1;
        int sA = 2 * g, sB = 2 * g + 1;
        uint32_t scA, mA, scB, mB;
        if (sA < 4) { scA = byte(sA) & 63; mA = byte(sA + 4) & 63; }
        else { scA = (byte(sA + 4) & 0xF) | ((byte(sA - 4) >> 6) << 4); mA = (byte(sA + 4) >> 4) | ((byte(sA) >> 6) << 4); }
        if (sB < 4) { scB = byte(sB) & 63; mB = byte(sB + 4) & 63; }
        else { scB = (byte(sB + 4) & 0xF) | ((byte(sB - 4) >> 6) << 4); mB = (byte(sB + 4) >> 4) | ((byte(sB) >> 6) << 4); }
        float d = h2f((uint16_t)(hdr.x & 0xFFFF)), dmin = h2f((uint16_t)(hdr.x >> 16));
        float al = 0.f, ah = 0.f;
        const uint32_t q[4] = {qs.x, qs.y, qs.z, qs.w};
#pragma unroll
        for (int w = 0; w < 4; w++) {
            QRM_DOT4(q[w] & 0x0F0F0F0Fu, xu.x, 4 * w, al, 16);
            QRM_DOT4(q[w] & 0xF0F0F0F0u, xu.x, 16 + 4 * w, ah, 15);
        }
        float sxl = xu.s[0] + xu.s[1], sxh = xu.s[2] + xu.s[3];
        float qxl = 64.f * (al - 2.f * sxl);
        float qxh = 8.f * (ah - 2.f * sxh);
        return d * ((float)scA * qxl + (float)scB * qxh) - dmin * ((float)mA * sxl + (float)mB * sxh);
    }
};

// Q4_0 (split): qs[nb][16] | d[nb]; unit = one block (low nibble = weight i,
// high nibble = weight i+16, y = d*(q-8)).
template <> struct WUnit<Q4_0> {
    uint4 qs;
    uint16_t dh;
    __device__ __forceinline__ void load(const MatDev& m, int row, int u) {
        size_t blk = (size_t)row * (m.cols >> 5) + u;
        qs = ld_stream16(m.base + blk * 16);
        dh = ld_u16(m.base + m.nb * 16 + blk * 2);
    }
    __device__ __forceinline__ float dot(const XUnit& xu) const {
        float al = 0.f, ah = 0.f;
        const uint32_t q[4] = {qs.x, qs.y, qs.z, qs.w};
#pragma unroll
        for (int w = 0; w < 4; w++) {
            QRM_DOT4(q[w] & 0x0F0F0F0Fu, xu.x, 4 * w, al, 16);
            QRM_DOT4(q[w] & 0xF0F0F0F0u, xu.x, 16 + 4 * w, ah, 15);
        }
        float sxl = xu.s[0] + xu.s[1], sxh = xu.s[2] + xu.s[3];
        float qx = 64.f * (al - 2.f * sxl) + 8.f * (ah - 2.f * sxh);
        return h2f(dh) * (qx - 8.f * (sxl + sxh));
    }
};

// Q8_0 (split): qs[nb][32] | d[nb]; y = d*q, q int8.
template <> struct WUnit<Q8_0> {
    uint4 q0, q1;
    uint16_t dh;
    __device__ __forceinline__ void load(const MatDev& m, int row, int u) {
        size_t blk = (size_t)row * (m.cols >> 5) + u;
        q0 = ld_stream16(m.base + blk * 32);
        q1 = ld_stream16(m.base + blk * 32 + 16);
        dh = ld_u16(m.base + m.nb * 32 + blk * 2);
    }
    __device__ __forceinline__ float dot(const XUnit& xu) const {
        // b = q + 128 as an unsigned byte at POS 15: F = 2 + b/128 = 3 + q/128
        // -> sum q x = 128*(sum F x - 3 sum x)
        const uint32_t q[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
        float a = 0.f;
#pragma unroll
        for (int w = 0; w < 8; w++) QRM_DOT4(q[w] ^ 0x80808080u, xu.x, 4 * w, a, 15);
        float sx = (xu.s[0] + xu.s[1]) + (xu.s[2] + xu.s[3]);
        return h2f(dh) * (128.f * (a - 3.f * sx));
    }
};

// Q6_K (split): ql[nb][128] | qh[nb][64] | sc[nb][16] | d[nb].
// Unit uu (0..7) of a block: half h = uu/4, l in [8*(uu&3), +8):
// q1..q4 -> weights 128h + l + {0,32,64,96} with scales sc[8h + l/16 + {0,2,4,6}].
template <> struct WUnit<Q6_K> {
    uint2 a, b, hb, sc;
    uint16_t dh;
    int is;
    __device__ __forceinline__ void load(const MatDev& m, int row, int u) {
        size_t blk = (size_t)row * (m.cols >> 8) + (u >> 3);
        int uu = u & 7, h = uu >> 2, l0 = 8 * (uu & 3);
        const uint8_t* ql = m.base + blk * 128;
        a = ld_stream8(ql + 64 * h + l0);
        b = ld_stream8(ql + 64 * h + 32 + l0);
        hb = ld_stream8(m.base + m.nb * 128 + blk * 64 + 32 * h + l0);
        sc = __ldg((const uint2*)(m.base + m.nb * 192 + blk * 16 + 8 * h));
        dh = ld_u16(m.base + m.nb * 208 + blk * 2);
        is = (uu & 3) >> 1;
    }
    __device__ __forceinline__ float dot(const XUnit& xu) const {
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        const uint32_t A[2] = {a.x, a.y}, B[2] = {b.x, b.y}, H[2] = {hb.x, hb.y};
#pragma unroll
        for (int w = 0; w < 2; w++) {
            uint32_t q1 = (A[w] & 0x0F0F0F0Fu) | ((H[w] & 0x03030303u) << 4);
            uint32_t q2 = (B[w] & 0x0F0F0F0Fu) | (((H[w] >> 2) & 0x03030303u) << 4);
            uint32_t q3 = ((A[w] >> 4) & 0x0F0F0F0Fu) | (((H[w] >> 4) & 0x03030303u) << 4);
            uint32_t q4 = ((B[w] >> 4) & 0x0F0F0F0Fu) | (((H[w] >> 6) & 0x03030303u) << 4);
            QRM_DOT4(q1, xu.x, 0 + 4 * w, acc[0], 16);
            QRM_DOT4(q2, xu.x, 8 + 4 * w, acc[1], 16);
            QRM_DOT4(q3, xu.x, 16 + 4 * w, acc[2], 16);
            QRM_DOT4(q4, xu.x, 24 + 4 * w, acc[3], 16);
        }
        // sc bytes: [0..8) = sc[8h .. 8h+8); group g uses byte is + 2g (int8)
        float r = 0.f;
#pragma unroll
        for (int g = 0; g < 4; g++) {
            int byte = is + 2 * g;
            uint32_t w = byte < 4 ? sc.x : sc.y;
            int s8 = (int)(int8_t)((w >> (8 * (byte & 3))) & 0xFF);
            // sum (q-32) x = 64*sum F x - 160*sum x
            r += (float)s8 * (64.f * acc[g] - 160.f * xu.s[g]);
        }
        return h2f(dh) * r;
    }
};

// TRI (split): codes[nb][16] | scale[nb]; unit = half block (32 weights).
// Code c of weight i at bits 2(i&3) of byte i/4; value (c&1) - ((c>>1)&1)
// (01 -> +1, 10 -> -1, 00 and 11 -> 0), times the scale.
template <> struct WUnit<TRI> {
    uint2 c;
    uint16_t sh;
    __device__ __forceinline__ void load(const MatDev& m, int row, int u) {
        size_t blk = (size_t)row * (m.cols >> 6) + (u >> 1);
        c = ld_stream8(m.base + blk * 16 + 8 * (u & 1));
        sh = ld_u16(m.base + m.nb * 16 + blk * 2);
    }
    __device__ __forceinline__ float dot(const XUnit& xu) const {
        float p = 0.f, n = 0.f;
        const uint32_t W[2] = {c.x, c.y};
#pragma unroll
        for (int w = 0; w < 2; w++) {
#pragma unroll
            for (int i = 0; i < 16; i++) {
                uint32_t code = (W[w] >> (2 * i)) & 3u;
                float xv = xu.x[16 * w + i];
                p += (code & 1u) ? xv : 0.f;
                n += (code & 2u) ? xv : 0.f;
            }
        }
        return h2f(sh) * (p - n);
    }
};

// ---------------------------------------------------------------- raw formats
// Blocks exactly as stored in .qw (row r, block b at (r * blocks_per_row + b)
// * block bytes); fields are read with loads no wider than the block's
// alignment.  Each unit decodes its 32 weights to f32 (the decoder formulas of
// BlockDequantizer.cs) and accumulates w * x in f32.
__device__ __forceinline__ uint32_t ldb(const uint8_t* p) { return __ldg(p); }
__device__ __forceinline__ uint32_t ldh(const uint8_t* p) { return __ldg(reinterpret_cast<const unsigned short*>(p)); }
__device__ __forceinline__ uint32_t ldw(const uint8_t* p) { return __ldg(reinterpret_cast<const unsigned int*>(p)); }
template <int BB>
__device__ __forceinline__ const uint8_t* raw_block(const MatDev& m, int row, int u) {
    return m.base + ((size_t)row * (m.cols >> 8) + (u >> 3)) * BB;
}

// Q2_K (84 B: scales[16] | qs[64] | d | dmin; BlockDequantizer.cs:87-114):
// weight w: code (qs[32*(w/128) + w%32] >> 2*((w%128)/32)) & 3, sub-block
// w/16: y = d*(sc & 15)*q - dmin*(sc >> 4).  Unit uu covers sub-blocks 2uu, 2uu+1.
template <> struct WUnit<Q2_K> {
    uint32_t q[8], scw, dd;
    int uu;
    __device__ __forceinline__ void load(const MatDev& m, int row, int u) {
        const uint8_t* b = raw_block<84>(m, row, u);   // 84 = 4 x 21: 4-byte aligned
        uu = u & 7;
        const uint8_t* qs = b + 16 + 32 * (uu >> 2);
#pragma unroll
        for (int i = 0; i < 8; i++) q[i] = ldw(qs + 4 * i);
        scw = ldh(b + 2 * uu);                        // sc[2uu] | sc[2uu+1] << 8
        dd = ldw(b + 80);                             // d | dmin << 16
    }
    __device__ __forceinline__ float dot(const XUnit& xu) const {
        const int sh = 2 * (uu & 3);
        float a0 = 0.f, a1 = 0.f;
#pragma unroll
        for (int i = 0; i < 32; i++) {
            const float qv = (float)((q[i >> 2] >> (8 * (i & 3) + sh)) & 3u);
            if (i < 16) a0 = fmaf(qv, xu.x[i], a0);
            else a1 = fmaf(qv, xu.x[i], a1);
        }
        const float d = h2f((uint16_t)(dd & 0xFFFF)), dmin = h2f((uint16_t)(dd >> 16));
        const uint32_t s0 = scw & 0xFF, s1 = scw >> 8;
        return d * ((float)(s0 & 15) * a0 + (float)(s1 & 15) * a1) -
               dmin * ((float)(s0 >> 4) * (xu.s[0] + xu.s[1]) + (float)(s1 >> 4) * (xu.s[2] + xu.s[3]));
    }
};

// Q3_K (110 B: hmask[32] | qs[64] | scales[12] | d; BlockDequantizer.cs:117-151):
// code as Q2_K, minus 4 where hmask[w%32] lacks bit w/32; 16 signed 6-bit
// scales (kmask shuffle of the 12 packed bytes); y = d*sc*q.
template <> struct WUnit<Q3_K> {
    uint32_t q[8], hm[8];
    int sc0, sc1, uu;
    uint32_t dh;
    __device__ __forceinline__ void load(const MatDev& m, int row, int u) {
        const uint8_t* b = raw_block<110>(m, row, u);  // 2-byte aligned
        uu = u & 7;
        const uint8_t* qs = b + 32 + 32 * (uu >> 2);
#pragma unroll
        for (int i = 0; i < 8; i++) {
            q[i] = ldh(qs + 4 * i) | (ldh(qs + 4 * i + 2) << 16);
            hm[i] = ldh(b + 4 * i) | (ldh(b + 4 * i + 2) << 16);
        }
        // scales 2uu, 2uu+1 of the shuffle: index i -> word i/4 of (r0, r1, r2, r3)
        uint32_t a[3];
#pragma unroll
        for (int w = 0; w < 3; w++) a[w] = ldh(b + 96 + 4 * w) | (ldh(b + 96 + 4 * w + 2) << 16);
        auto scale = [&](int i) {
            const int g = i >> 2, by = i & 3;
            const uint32_t lo = g & 1 ? a[1] : a[0];
            const uint32_t nib = (g >= 2 ? (lo >> 4) : lo) & 0x0F0F0F0Fu;
            const uint32_t hi = (a[2] >> (2 * g)) & 0x03030303u;
            const uint32_t r = nib | (hi << 4);
            return (int)((r >> (8 * by)) & 0xFF) - 32;
        };
        sc0 = scale(2 * uu);
        sc1 = scale(2 * uu + 1);
        dh = ldh(b + 108);
    }
    __device__ __forceinline__ float dot(const XUnit& xu) const {
        const int sh = 2 * (uu & 3);
        float a0 = 0.f, a1 = 0.f;
#pragma unroll
        for (int i = 0; i < 32; i++) {
            int qv = (int)((q[i >> 2] >> (8 * (i & 3) + sh)) & 3u);
            if (((hm[i >> 2] >> (8 * (i & 3) + uu)) & 1u) == 0) qv -= 4;
            if (i < 16) a0 = fmaf((float)qv, xu.x[i], a0);
            else a1 = fmaf((float)qv, xu.x[i], a1);
        }
        return h2f((uint16_t)dh) * ((float)sc0 * a0 + (float)sc1 * a1);
    }
};

// Q5_K (176 B: d | dmin | scales[12] | ql[128] | qh[32]; BlockDequantizer.cs:
// 198-226): unit uu = sub-block uu; q = nibble (uu&1) of ql[32*(uu/2) + i]
// + 16 * bit uu of qh[i]; y = d*sc*q - dmin*m (GetScaleMinK4).
template <> struct WUnit<Q5_K> {
    uint4 hdr, l0, l1, h0, h1;
    int uu;
    __device__ __forceinline__ void load(const MatDev& m, int row, int u) {
        const uint8_t* b = raw_block<176>(m, row, u);  // 176 = 16 x 11: 16-byte aligned
        uu = u & 7;
        hdr = __ldg(reinterpret_cast<const uint4*>(b));
        const uint8_t* ql = b + 16 + 32 * (uu >> 1);
        l0 = ld_stream16(ql);
        l1 = ld_stream16(ql + 16);
        h0 = __ldg(reinterpret_cast<const uint4*>(b + 144));
        h1 = __ldg(reinterpret_cast<const uint4*>(b + 160));
    }
    __device__ __forceinline__ float dot(const XUnit& xu) const {
        const uint32_t L[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
        const uint32_t H[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
        const int ls = 4 * (uu & 1);
        float a = 0.f;
#pragma unroll
        for (int i = 0; i < 32; i++) {
            const uint32_t qv = ((L[i >> 2] >> (8 * (i & 3) + ls)) & 15u) + 16u * ((H[i >> 2] >> (8 * (i & 3) + uu)) & 1u);
            a = fmaf((float)qv, xu.x[i], a);
        }
        // GetScaleMinK4 (BlockDequantizer.cs:155-166) on scale bytes 4..15 of the block
        const uint32_t sw[3] = {hdr.y, hdr.z, hdr.w};
        auto byte = [&](int i) -> uint32_t { return (sw[i >> 2] >> (8 * (i & 3))) & 0xFF; };
        uint32_t sc, mn;
        if (uu < 4) { sc = byte(uu) & 63; mn = byte(uu + 4) & 63; }
        else { sc = (byte(uu + 4) & 0xF) | ((byte(uu - 4) >> 6) << 4); mn = (byte(uu + 4) >> 4) | ((byte(uu) >> 6) << 4); }
        const float d = h2f((uint16_t)(hdr.x & 0xFFFF)), dmin = h2f((uint16_t)(hdr.x >> 16));
        return d * (float)sc * a - dmin * (float)mn * ((xu.s[0] + xu.s[1]) + (xu.s[2] + xu.s[3]));
    }
};

// I8_BLK (258 B: d | int8 q[256]; BlockDequantizer.cs:278-290): y = d*q.
template <> struct WUnit<I8_BLK> {
    uint32_t q[8];
    uint32_t dh;
    __device__ __forceinline__ void load(const MatDev& m, int row, int u) {
        const uint8_t* b = raw_block<258>(m, row, u);  // 2-byte aligned
        const uint8_t* qs = b + 2 + 32 * (u & 7);
#pragma unroll
        for (int i = 0; i < 8; i++) q[i] = ldh(qs + 4 * i) | (ldh(qs + 4 * i + 2) << 16);
        dh = ldh(b);
    }
    __device__ __forceinline__ float dot(const XUnit& xu) const {
        float a = 0.f;
#pragma unroll
        for (int i = 0; i < 32; i++) a = fmaf((float)(int8_t)((q[i >> 2] >> (8 * (i & 3))) & 0xFF), xu.x[i], a);
        return h2f((uint16_t)dh) * a;
    }
};

// B1 (34 B: f16 a | sign mask[32]; BlockDequantizer.cs:299-313): y = +a where
// bit i of the mask is set, else -a.  B1X (47 B) adds k <= 4 exact values
// (u8 idx, f16 v) at byte 35 (BlockDequantizer.cs:315-336).
template <int FMT, int BB>
struct WUnitB1 {
    uint32_t mask, ah;
    int uu, k;
    uint32_t ex[4];   // idx | v << 16 of the block's exceptions (B1X)
    __device__ __forceinline__ void load(const MatDev& m, int row, int u) {
        const uint8_t* b = raw_block<BB>(m, row, u);
        uu = u & 7;
        const uint8_t* mk = b + 2 + 4 * uu;
        mask = ldb(mk) | (ldb(mk + 1) << 8) | (ldb(mk + 2) << 16) | (ldb(mk + 3) << 24);
        ah = ldb(b) | (ldb(b + 1) << 8);
        k = 0;
        if (FMT == B1X) {
            k = min((int)ldb(b + 34), 4);
            for (int e = 0; e < k; e++) {
                const uint8_t* p = b + 35 + 3 * e;
                ex[e] = ldb(p) | (ldb(p + 1) << 16) | (ldb(p + 2) << 24);
            }
        }
    }
    __device__ __forceinline__ float dot(const XUnit& xu) const {
        float pos = 0.f;
#pragma unroll
        for (int i = 0; i < 32; i++) pos += ((mask >> i) & 1u) ? xu.x[i] : 0.f;
        const float sx = (xu.s[0] + xu.s[1]) + (xu.s[2] + xu.s[3]);
        const float a = h2f((uint16_t)ah);
        float r = a * (2.f * pos - sx);
        for (int e = 0; e < k; e++) {
            const int idx = (int)(ex[e] & 0xFF) - 32 * uu;
            if (idx < 0 || idx >= 32) continue;
            const float v = h2f((uint16_t)(ex[e] >> 16));
            float xv = 0.f;
#pragma unroll
            for (int i = 0; i < 32; i++) xv = i == idx ? xu.x[i] : xv;
            r += (v - (((mask >> idx) & 1u) ? a : -a)) * xv;
        }
        return r;
    }
};
template <> struct WUnit<B1> : WUnitB1<B1, 34> {};
template <> struct WUnit<B1X> : WUnitB1<B1X, 47> {};

// T1E / T1E_LO (u16 n0 | u16 nP | f16 a | rANS stream of SB bytes;
// BlockDequantizer.cs:338-359, EntropyCoder.Decode3, EntropyCoder.cs:83-110):
// symbols 0 -> 0, 1 -> +a, 2 -> -a.  The stream decodes front to back, so the
// unit decodes symbols 0 .. 32uu+31 and keeps its 32.  A corrupt stream (one
// the reference's decoder rejects: it would read past its bytes, or decode a
// zero-frequency symbol) gives some finite values; every loop stays bounded.
template <int SB>
struct WUnitT1E {
    const uint8_t* b;
    int uu;
    __device__ __forceinline__ void load(const MatDev& m, int row, int u) {
        b = raw_block<6 + SB>(m, row, u);
        uu = u & 7;
    }
    __device__ __forceinline__ float dot(const XUnit& xu) const {
        const uint32_t f0 = ldb(b) | (ldb(b + 1) << 8), f1 = ldb(b + 2) | (ldb(b + 3) << 8);
        const float a = h2f((uint16_t)(ldb(b + 4) | (ldb(b + 5) << 8)));
        const uint32_t f2 = 256u - f0 - f1, L = 1u << 23;
        const uint8_t* src = b + 6;
        int p = 0;
        uint32_t x = 0;
        for (int i = 0; i < 4; i++) x = (x << 8) | (p < SB ? ldb(src + p++) : 0u);
        uint32_t pm = 0, nm = 0;   // this unit's +a and -a weights
        const int first = 32 * uu;
        for (int i = 0; i < first + 32; i++) {
            while (x < L) {
                if (p >= SB + 4) { x = L; break; }   // past the stream: corrupt
                x = (x << 8) | (p < SB ? ldb(src + p) : 0u);
                p++;
            }
            const uint32_t slot = x & 255u;
            uint32_t s, f, c;
            if (slot < f0) { s = 0; f = f0; c = 0; }
            else if (slot < f0 + f1) { s = 1; f = f1; c = f0; }
            else { s = 2; f = f2; c = f0 + f1; }
            if (f == 0 || f > 256u) break;        // corrupt: zero-frequency symbol or bad counts
            x = f * (x >> 8) + slot - c;
            if (i >= first) {
                if (s == 1) pm |= 1u << (i - first);
                else if (s == 2) nm |= 1u << (i - first);
            }
        }
        float pos = 0.f, neg = 0.f;
#pragma unroll
        for (int q = 0; q < 32; q++) {
            pos += ((pm >> q) & 1u) ? xu.x[q] : 0.f;
            neg += ((nm >> q) & 1u) ? xu.x[q] : 0.f;
        }
        return a * (pos - neg);
    }
};
template <> struct WUnit<T1E> : WUnitT1E<34> {};
template <> struct WUnit<T1E_LO> : WUnitT1E<26> {};

// ------------------------------------------------------------ reduction

// Transposing warp reduction of NV (power of two, <= 32) values: afterwards
// lane l holds the warp sum of value index  vidx(l) = sum over stages of
// bit(l, 16>>s) * (NV >> (s+1)).  Values are reduced in a fixed order.
template <int NV>
__device__ __forceinline__ float warp_reduce_transposed(float (&v)[NV], int lane) {
    int n = NV;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        if (n > 1) {
            const bool upper = (lane & o) != 0;
#pragma unroll
            for (int i = 0; i < NV / 2; i++) {
                if (i < n / 2) {
                    float send = upper ? v[i] : v[i + n / 2];
                    float keep = upper ? v[i + n / 2] : v[i];
                    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
                }
            }
            n >>= 1;
        } else {
            v[0] += __shfl_xor_sync(0xffffffffu, v[0], o);
        }
    }
    return v[0];
}
template <int NV>
__device__ __forceinline__ int transposed_index(int lane) {
    int idx = 0, n = NV;
#pragma unroll
    for (int o = 16; o > 0 && n > 1; o >>= 1) {
        if (lane & o) idx += n / 2;
        n >>= 1;
    }
    return idx;
}
// lane that writes value index v (the lowest lane holding it)
template <int NV>
__device__ __forceinline__ bool transposed_writer(int lane) {
    // lanes differing only in bits below the last transposing stage hold copies
    constexpr int kStages = NV >= 32 ? 5 : NV >= 16 ? 4 : NV >= 8 ? 3 : NV >= 4 ? 2 : NV >= 2 ? 1 : 0;
    constexpr int kLowMask = (1 << (5 - kStages)) - 1;
    return (lane & kLowMask) == 0;
}

// ------------------------------------------------------------ kernels

struct GemvParams {
    const MatDev* mats;        // [E+1][3]: gate, up, down; row E = shared expert
    const int32_t* active;     // slot -> expert (E = shared)
    const int32_t* offsets;    // [E+1]
    const int32_t* perm;       // [T*k]
    const int32_t* pos_tok;    // [T*k] token of the assignment at each position (perm / k)
    const int4* slot_info;     // [slots] (expert, first position, tokens, first token), or null
    const int32_t* n_active;   // routed slots (written by the dispatch kernel)
    int32_t* ctr;              // work counter of this launch (zeroed before it)
    const float* x_routed;     // gate/up: xn [T x d]; down: h [T*k x f]
    const float* x_shared;     // gate/up: xn; down: hs [T x f]
    float* out_routed;         // gate/up: h [T*k x f]; down: y [T*k x d]
    float* out_shared;         // gate/up: hs [T x f]; down: ys [T x d]
    int T, k, E;
    int T_sh;                  // shared-expert tokens (rows of x_shared / out_shared)
    int rows, cols, tiles;     // per expert matrix
    float limit;               // SwiGLU limit (<= 0: plain)
    int routed_by_token;       // gate/up: routed inputs are token rows (perm/k)
    int mode;                  // 0: routed + shared slots, 1: routed only, 2: shared only
    int has_shared;
    // quantised activation tables (integer tensor-core kernel): routed rows are
    // token rows (gate/up, row = perm/k) or assignment rows (down, row = off+i);
    // shared rows follow at xtab_shared_base
    const uint8_t* xtab;
    int xtab_stride;
    int xtab_shared_base;
    int xtab_rows;             // table rows written for this launch
    // when set, the kernel builds resident tables itself from these f32 rows
    // (rows < xq_split from xq_a, the rest from xq_b) instead of copying xtab
    const float* xq_a;
    const float* xq_b;
    int xq_split;
    // expert parallelism over peer memory, down launches of the streaming
    // kernel: every routed output row goes straight into its owner's mailbox
    // (gathered token u = q*ep_T + t, slot j -> row t*k + j of owner q's y
    // block) and the last consumer warp of the grid raises this rank's output
    // flag in every owner's mailbox (null ep_base: rows stay in out_routed)
    const unsigned long long* ep_base;   // [ep_G] mailboxes, mapped here
    long long ep_y, ep_flag;             // mailbox offsets of the y block and the output flags
    const uint32_t* ep_epoch;            // this forward's epoch (advanced by its dispatch)
    uint32_t* ep_cnt;                    // consumer warps done (zero between launches)
    int ep_G, ep_rank, ep_T;
    // launched as a programmatic dependent: 1 = wait for the predecessor
    // before anything, 2 = the producer streams weights before the wait (the
    // routing it reads was final two launches earlier; only the activations
    // come from the predecessor)
    int pdl;
};

__device__ __forceinline__ float swiglu(float g, float u, float limit) {
    if (limit > 0.f) {
        // Glm5Ops.LimitedSwiglu (Glm5Ops.cs:243-256)
        g = g > limit ? limit : g;
        u = u > limit ? limit : (u < -limit ? -limit : u);
    }
    // TransformerOps.Silu / SiluMulInPlace: g / (1 + exp(-g)) * u
    return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.f, expf_glibc(-g))), u);
}

// M = matrices per item (2: gate+up -> SwiGLU, 1: down), R = rows per tile,
// NT = tokens per pass.
constexpr int kGemvMaxThreads = 512;   // rows up to 16384 columns (512 units)

template <int FMT, int M, int R, int NT>
__global__ void __launch_bounds__(kGemvMaxThreads)
expert_gemv_kernel(GemvParams p) {
    constexpr int NV = M * R * NT;
    static_assert(NV <= 32 && (NV & (NV - 1)) == 0, "NV must be a power of two <= 32");
    __shared__ float red[32][NV];
    __shared__ int s_item[2];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nwarps = blockDim.x >> 5;
    const int U = p.cols >> 5;
    const int u = tid;
    const bool has_unit = u < U;
    const int n_active = *p.n_active;
    const int n_items = p.mode == 2 ? (p.has_shared ? p.tiles : 0)
                                    : (n_active + (p.mode == 0 && p.has_shared ? 1 : 0)) * p.tiles;
    const int slot_base = p.mode == 2 ? n_active : 0;
    int it = 0;
    for (;;) {
        if (tid == 0) s_item[it & 1] = blockIdx.x + it * gridDim.x;   // static striding
        __syncthreads();
        const int item = s_item[it & 1];
        it++;
        if (item >= n_items) break;
        const int sl = item / p.tiles, tile = item - sl * p.tiles;
        const int slot = slot_base + sl;
        const int e = p.active[slot];
        const bool shared = slot >= n_active;
        const int r0 = tile * R;
        int n_tok, off = 0;
        if (shared) n_tok = p.T_sh;
        else { off = p.offsets[e]; n_tok = p.offsets[e + 1] - off; }
        const MatDev* md = p.mats + (size_t)e * 3;
        MatDev mat[M];
#pragma unroll
        for (int m = 0; m < M; m++) mat[m] = md[M == 2 ? m : 2];

        WUnit<FMT> w[M][R];
        if (has_unit) {
#pragma unroll
            for (int m = 0; m < M; m++)
#pragma unroll
                for (int rr = 0; rr < R; rr++) {
                    int row = min(r0 + rr, p.rows - 1);
                    w[m][rr].load(mat[m], row, u);
                }
        }
        for (int t0 = 0; t0 < n_tok; t0 += NT) {
            float acc[NV];
#pragma unroll
            for (int i = 0; i < NV; i++) acc[i] = 0.f;
            if (has_unit) {
#pragma unroll
                for (int t = 0; t < NT; t++) {
                    if (t0 + t < n_tok) {
                        const float* xrow;
                        if (shared) xrow = p.x_shared + (size_t)(t0 + t) * p.cols;
                        else if (p.routed_by_token) xrow = p.x_routed + (size_t)(p.perm[off + t0 + t] / p.k) * p.cols;
                        else xrow = p.x_routed + (size_t)(off + t0 + t) * p.cols;
                        XUnit xu;
                        load_x<FMT>(xu, xrow, u);
#pragma unroll
                        for (int m = 0; m < M; m++)
#pragma unroll
                            for (int rr = 0; rr < R; rr++) acc[(m * R + rr) * NT + t] = w[m][rr].dot(xu);
                    }
                }
            }
            float v = warp_reduce_transposed<NV>(acc, lane);
            if (transposed_writer<NV>(lane)) red[warp][transposed_index<NV>(lane)] = v;
            __syncthreads();
            if (tid < NV) {
                float s = 0.f;
                for (int wi = 0; wi < nwarps; wi++) s += red[wi][tid];
                red[0][tid] = s;  // safe: only thread tid reads/writes column tid
            }
            __syncthreads();
            if (tid < R * NT) {
                const int rr = tid / NT, t = tid - rr * NT;
                const int row = r0 + rr;
                if (row < p.rows && t0 + t < n_tok) {
                    float res;
                    if (M == 2) res = swiglu(red[0][(0 * R + rr) * NT + t], red[0][(1 * R + rr) * NT + t], p.limit);
                    else res = red[0][rr * NT + t];
                    float* orow = shared ? p.out_shared + (size_t)(t0 + t) * p.rows
                                         : p.out_routed + (size_t)(off + t0 + t) * p.rows;
                    orow[row] = res;
                }
            }
            __syncthreads();
        }
    }
}

}  // namespace qrm
