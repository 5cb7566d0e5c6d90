// oracle.cpp -- CPU restatement of QuantRunner's MoE FFN hot path.
//
// TEST INFRASTRUCTURE ONLY (parity checker and timed CPU baseline); the
// product never links it.  Build flags: -O3 -ffp-contract=off, no fast-math,
// so every C# float operation below is one IEEE-754 binary32 operation in the
// same order as the reference.  See oracle.h for the contract.
#include "oracle.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <thread>
#include <vector>

namespace {

inline float u2f(uint32_t u) { float f; std::memcpy(&f, &u, 4); return f; }
inline uint32_t f2u(float f) { uint32_t u; std::memcpy(&u, &f, 4); return u; }
inline uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

// C# (int) cast of a float on x64: truncation, 0x80000000 when out of range.
inline int cs_int(float v) {
    if (!(v > -2147483904.0f && v < 2147483648.0f)) return INT32_MIN;
    return (int)v;
}
// MathF.Round: round half to even.
inline float cs_round(float v) { return std::rint(v); }
// BlockQuantizer.ClampQ, BlockQuantizer.cs:760
inline int clampq(int v, int lo, int hi) { return v < lo ? lo : v > hi ? hi : v; }

}  // namespace

extern "C" {

// ------------------------------------------------------------------ Dtypes.cs

int orc_block_spec(int fmt, int* bs, int* bb) {
    // Dtypes.BlockSpec, Dtypes.cs:38-57
    int s, b;
    switch (fmt) {
        case ORC_F32: s = 1; b = 4; break;
        case ORC_F16: s = 1; b = 2; break;
        case ORC_BF16: s = 1; b = 2; break;
        case ORC_Q4_0: s = 32; b = 20; break;
        case ORC_Q8_0: s = 32; b = 34; break;
        case ORC_Q4_K: s = 256; b = 144; break;
        case ORC_Q6_K: s = 256; b = 210; break;
        case ORC_TRI: s = 64; b = 18; break;
        case ORC_Q2_K: s = 256; b = 84; break;
        case ORC_Q3_K: s = 256; b = 110; break;
        case ORC_Q5_K: s = 256; b = 176; break;
        case ORC_I8_BLK: s = 256; b = 258; break;
        case ORC_B1: s = 256; b = 34; break;
        case ORC_B1X: s = 256; b = 47; break;
        case ORC_T1E: s = 256; b = 40; break;
        case ORC_T1E_LO: s = 256; b = 32; break;
        default: return -1;
    }
    if (bs) *bs = s;
    if (bb) *bb = b;
    return 0;
}

int64_t orc_tensor_bytes(int64_t n, int fmt) {
    // Dtypes.TensorBytes, Dtypes.cs:60-65
    int bs, bb;
    if (orc_block_spec(fmt, &bs, &bb) != 0 || n % bs != 0) return -1;
    return n / bs * bb;
}

float orc_f16_to_f32(uint16_t h) {
    // Dtypes.F16ToFloat, Dtypes.cs:76-97
    uint32_t sign = (uint32_t)(h & 0x8000) << 16;
    uint32_t exp = (uint32_t)(h >> 10) & 0x1F;
    uint32_t man = (uint32_t)(h & 0x3FF);
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {
            int e = -1;
            uint32_t m = man;
            do { m <<= 1; e++; } while ((m & 0x400) == 0);
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((m & 0x3FF) << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7F800000u | (man << 13);
    } else {
        bits = sign | ((exp + 112) << 23) | (man << 13);
    }
    return u2f(bits);
}

uint16_t orc_f32_to_f16(float f) {
    // Dtypes.FloatToF16, Dtypes.cs:100-126: mantissa rounds half-up (+0x1000)
    // for normals, nearest-even for subnormals.
    uint32_t x = f2u(f);
    uint32_t sign = (x >> 16) & 0x8000u;
    int exp = (int)((x >> 23) & 0xFF) - 127;
    uint32_t man = x & 0x7FFFFF;
    if (((x >> 23) & 0xFF) == 0xFF) return (uint16_t)(sign | 0x7C00u | (man != 0 ? 0x200u : 0u));
    if (exp > 15) return (uint16_t)(sign | 0x7C00u);
    if (exp >= -14) {
        uint32_t rounded = man + 0x1000u;
        if ((rounded & 0x800000u) != 0) { rounded = 0; exp++; }
        return (uint16_t)(sign | ((uint32_t)(exp + 15) << 10) | (rounded >> 13));
    }
    if (exp < -25) return (uint16_t)sign;
    uint32_t bits23 = 0x800000u | man;
    int shift = (-exp - 14) + 13;
    uint32_t half = bits23 >> shift;
    uint32_t rem = bits23 & ((1u << shift) - 1);
    uint32_t mid = 1u << (shift - 1);
    if (rem > mid || (rem == mid && (half & 1) != 0)) half++;
    return (uint16_t)(sign | half);
}

float orc_bf16_to_f32(uint16_t b) { return u2f((uint32_t)b << 16); }  // Dtypes.cs:129

uint16_t orc_f32_to_bf16(float f) {
    // Dtypes.FloatToBf16, Dtypes.cs:132-139
    uint32_t x = f2u(f);
    uint32_t lsb = (x >> 16) & 1;
    x += 0x7FFFu + lsb;
    return (uint16_t)(x >> 16);
}

void orc_f32_to_f16_batch(const float* x, uint16_t* y, int64_t n) {
    for (int64_t i = 0; i < n; i++) y[i] = orc_f32_to_f16(x[i]);
}

// ------------------------------------------------------------ BlockQuantizer

static void put16(uint8_t* p, uint16_t v) { p[0] = (uint8_t)(v & 0xFF); p[1] = (uint8_t)(v >> 8); }

static void quant_q4_0(const float* x, int64_t n, uint8_t* y) {
    // BlockQuantizer.QuantizeQ4_0, BlockQuantizer.cs:69-93
    int64_t nb = n / 32;
    for (int64_t b = 0; b < nb; b++, x += 32, y += 20) {
        float amax = 0.f;
        for (int i = 0; i < 32; i++) { float a = std::fabs(x[i]); if (a > amax) amax = a; }
        float d = amax / 8.f;
        put16(y, orc_f32_to_f16(d));
        if (d == 0.f) { for (int i = 0; i < 16; i++) y[2 + i] = 8; continue; }
        float id = 1.f / d;
        for (int i = 0; i < 16; i++) {
            int q0 = clampq(cs_int(cs_round(x[i] * id)) + 8, 0, 15);
            int q1 = clampq(cs_int(cs_round(x[i + 16] * id)) + 8, 0, 15);
            y[2 + i] = (uint8_t)(q0 | (q1 << 4));
        }
        // bytes 18-19 are never written by the reference; the .qw buffers it
        // fills start zeroed, so they stay 0 here too.
        y[18] = 0; y[19] = 0;
    }
}

static void quant_q8_0(const float* x, int64_t n, uint8_t* y) {
    // BlockQuantizer.QuantizeQ8_0, BlockQuantizer.cs:97-116
    int64_t nb = n / 32;
    for (int64_t b = 0; b < nb; b++, x += 32, y += 34) {
        float amax = 0.f;
        for (int i = 0; i < 32; i++) { float a = std::fabs(x[i]); if (a > amax) amax = a; }
        float d = amax / 127.f;
        put16(y, orc_f32_to_f16(d));
        if (d == 0.f) { for (int i = 0; i < 32; i++) y[2 + i] = 0; continue; }
        float id = 1.f / d;
        for (int i = 0; i < 32; i++) y[2 + i] = (uint8_t)(int8_t)clampq(cs_int(cs_round(x[i] * id)), -128, 127);
    }
}

static void quant_q4_k(const float* x, int64_t n, uint8_t* y) {
    // BlockQuantizer.QuantizeQ4_K, BlockQuantizer.cs:248-318.  L[] lives for
    // the whole call, as the reference's stackalloc does: a sub-block whose
    // scale rounds to 0 keeps the previous block's codes.
    int64_t nb = n / 256;
    float mins[8], maxs[8];
    int L[256] = {0};
    int sc[8], m[8];
    uint8_t q[12];
    for (int64_t b = 0; b < nb; b++, x += 256, y += 144) {
        float amax = 0.f, amink = 0.f;
        for (int s = 0; s < 8; s++) {
            float mn = 3.40282347e+38f, mx = -3.40282347e+38f;
            for (int i = 0; i < 32; i++) {
                float v = x[s * 32 + i];
                if (v < mn) mn = v;
                if (v > mx) mx = v;
            }
            if (mn > 0) mn = 0;
            mins[s] = mn; maxs[s] = mx;
            float range = mx - mn;
            if (range > amax) amax = range;
            if (-mn > amink) amink = -mn;
        }
        std::memset(y, 0, 144);
        if (amax <= 0.f) continue;
        float d = amax / 945.f, dmin = amink > 0 ? amink / 63.f : 0.f;
        put16(y, orc_f32_to_f16(d));
        put16(y + 2, orc_f32_to_f16(dmin));
        float iscale = 63.f / amax, ismin = dmin > 0 ? 63.f / amink : 0.f;
        for (int s = 0; s < 8; s++) {
            sc[s] = clampq(cs_int(cs_round(iscale * (maxs[s] - mins[s]))), 0, 63);
            m[s] = dmin > 0 ? clampq(cs_int(cs_round(ismin * (-mins[s]))), 0, 63) : 0;
        }
        for (int j = 0; j < 4; j++) {
            q[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
            q[j + 4] = (uint8_t)((m[j] & 63) | ((m[j + 4] >> 4) << 6));
            q[j + 8] = (uint8_t)((sc[j + 4] & 0xF) | ((m[j + 4] & 0xF) << 4));
        }
        for (int i = 0; i < 12; i++) y[4 + i] = q[i];
        for (int s = 0; s < 8; s++) {
            float a = d * sc[s], bias = dmin * m[s];
            if (a <= 0.f) continue;
            for (int i = 0; i < 32; i++)
                L[s * 32 + i] = clampq(cs_int(cs_round((x[s * 32 + i] + bias) / a)), 0, 15);
        }
        for (int s = 0; s < 8; s++) {
            int baseByte = 16 + (s / 2) * 32;
            int nibbleHi = s & 1;
            for (int i = 0; i < 32; i++) {
                int val = L[s * 32 + i];
                if (nibbleHi == 0) y[baseByte + i] |= (uint8_t)val;
                else y[baseByte + i] |= (uint8_t)(val << 4);
            }
        }
    }
}

static void quant_q6_k(const float* x, int64_t n, uint8_t* y) {
    // BlockQuantizer.QuantizeQ6_K, BlockQuantizer.cs:398-446
    int64_t nb = n / 256;
    float subAmax[16];
    int sc[16];
    for (int64_t b = 0; b < nb; b++, x += 256, y += 210) {
        float amax = 0.f;
        for (int s = 0; s < 16; s++) {
            float mx = 0.f;
            for (int i = 0; i < 16; i++) { float a = std::fabs(x[s * 16 + i]); if (a > mx) mx = a; }
            subAmax[s] = mx;
            if (mx > amax) amax = mx;
        }
        std::memset(y, 0, 210);
        if (amax <= 0.f) continue;
        float d = amax / (31.f * 31.f);
        put16(y + 208, orc_f32_to_f16(d));
        for (int s = 0; s < 16; s++)
            sc[s] = clampq(cs_int(cs_round(subAmax[s] / (31.f * d))), subAmax[s] > 0 ? 1 : 0, 127);
        for (int w = 0; w < 256; w++) {
            int s = w / 16;
            float a = d * sc[s];
            int q = a > 0 ? clampq(cs_int(cs_round(x[w] / a)) + 32, 0, 63) : 32;
            int lo = q & 0xF, hi = (q >> 4) & 3;
            int nn = (w / 128) * 128;
            int r = w - nn;
            int slot = r / 32, l = r % 32;
            switch (slot) {
                case 0: y[nn / 2 + l] |= (uint8_t)lo; break;
                case 1: y[nn / 2 + l + 32] |= (uint8_t)lo; break;
                case 2: y[nn / 2 + l] |= (uint8_t)(lo << 4); break;
                case 3: y[nn / 2 + l + 32] |= (uint8_t)(lo << 4); break;
            }
            y[128 + nn / 4 + l] |= (uint8_t)(hi << (2 * slot));
        }
        for (int s = 0; s < 16; s++) y[192 + s] = (uint8_t)(int8_t)sc[s];
    }
}

static void quant_tri(const float* x, int64_t n, uint8_t* y) {
    // BlockQuantizer.QuantizeTri, BlockQuantizer.cs:456-521
    int64_t nb = n / 64;
    float sorted[64];
    for (int64_t b = 0; b < nb; b++, x += 64, y += 18) {
        std::memset(y, 0, 18);
        double energy = 0;
        float amax = 0.f;
        for (int i = 0; i < 64; i++) {
            float a = std::fabs(x[i]);
            sorted[i] = a;
            energy += a * (double)a;
            if (a > amax) amax = a;
        }
        if (amax == 0.f) continue;
        std::sort(sorted, sorted + 64);
        double bestErr = 1.7976931348623157e308;
        float bestT = 0.f, bestAlpha = amax;
        for (int j = 0; j <= 60; j += 4) {
            float t = sorted[j];
            double sum = 0;
            int kept = 0;
            for (int i = 0; i < 64; i++)
                if (std::fabs(x[i]) > t) { sum += std::fabs(x[i]); kept++; }
            if (kept == 0) continue;
            float alpha = (float)(sum / kept);
            double err = energy - 2.0 * alpha * sum + (double)alpha * alpha * kept;
            if (err < bestErr) { bestErr = err; bestT = t; bestAlpha = alpha; }
        }
        {
            double sumAll = 0;
            for (int i = 0; i < 64; i++) sumAll += std::fabs(x[i]);
            float tLegacy = (float)(sumAll / 64) * 0.5f;
            double sum = 0;
            int kept = 0;
            for (int i = 0; i < 64; i++)
                if (std::fabs(x[i]) >= tLegacy) { sum += std::fabs(x[i]); kept++; }
            if (kept > 0) {
                float alpha = (float)(sum / kept);
                double err = energy - 2.0 * alpha * sum + (double)alpha * alpha * kept;
                if (err < bestErr) { bestErr = err; bestT = tLegacy - 1e-9f; bestAlpha = alpha; }
            }
        }
        put16(y, orc_f32_to_f16(bestAlpha));
        for (int i = 0; i < 64; i++) {
            float a = std::fabs(x[i]);
            int code = a > bestT ? (x[i] > 0 ? 1 : 2) : 0;
            y[2 + i / 4] |= (uint8_t)(code << (2 * (i & 3)));
        }
    }
}

static void quant_tri_legacy(const float* x, int64_t n, uint8_t* y) {
    // BlockQuantizer.QuantizeTriLegacy, BlockQuantizer.cs:525-550
    int64_t nb = n / 64;
    for (int64_t b = 0; b < nb; b++, x += 64, y += 18) {
        std::memset(y, 0, 18);
        double sum = 0;
        for (int i = 0; i < 64; i++) sum += std::fabs(x[i]);
        float scale = (float)(sum / 64);
        if (scale == 0.f) continue;
        put16(y, orc_f32_to_f16(scale));
        float iscale = 1.f / scale;
        for (int i = 0; i < 64; i++) {
            int v = cs_int(cs_round(x[i] * iscale));
            int code = v > 0 ? 1 : v < 0 ? 2 : 0;
            y[2 + i / 4] |= (uint8_t)(code << (2 * (i & 3)));
        }
    }
}

int orc_quantize(int fmt, const float* src, int64_t n, uint8_t* dst) {
    int bs, bb;
    int f = fmt == 108 ? ORC_TRI : fmt;
    if (orc_block_spec(f, &bs, &bb) != 0 || n % bs != 0) return -1;
    switch (fmt) {
        case ORC_F32: std::memcpy(dst, src, (size_t)n * 4); return 0;
        case ORC_F16: for (int64_t i = 0; i < n; i++) put16(dst + 2 * i, orc_f32_to_f16(src[i])); return 0;
        case ORC_BF16: for (int64_t i = 0; i < n; i++) put16(dst + 2 * i, orc_f32_to_bf16(src[i])); return 0;
        case ORC_Q4_0: quant_q4_0(src, n, dst); return 0;
        case ORC_Q8_0: quant_q8_0(src, n, dst); return 0;
        case ORC_Q4_K: quant_q4_k(src, n, dst); return 0;
        case ORC_Q6_K: quant_q6_k(src, n, dst); return 0;
        case ORC_TRI: quant_tri(src, n, dst); return 0;
        case 108: quant_tri_legacy(src, n, dst); return 0;
        default: return -1;
    }
}

// ---------------------------------------------------------- BlockDequantizer

static inline void scale_min_k4(int j, const uint8_t* q, int* sc, int* m) {
    // BlockDequantizer.GetScaleMinK4, BlockDequantizer.cs:155-166
    if (j < 4) {
        *sc = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        *m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

// Q3_K's 16 signed 6-bit scales from the 12 packed bytes (the kmask shuffle
// over three little-endian words), BlockDequantizer.cs:130-143, DotKernels.cs:287-298
static void q3k_scales(const uint8_t* packed, int* sc) {
    uint32_t a0 = (uint32_t)(packed[0] | (packed[1] << 8) | (packed[2] << 16) | ((uint32_t)packed[3] << 24));
    uint32_t a1 = (uint32_t)(packed[4] | (packed[5] << 8) | (packed[6] << 16) | ((uint32_t)packed[7] << 24));
    uint32_t a2 = (uint32_t)(packed[8] | (packed[9] << 8) | (packed[10] << 16) | ((uint32_t)packed[11] << 24));
    uint32_t tmp = a2;
    uint32_t r2 = ((a0 >> 4) & 0x0f0f0f0fu) | (((tmp >> 4) & 0x03030303u) << 4);
    uint32_t r3 = ((a1 >> 4) & 0x0f0f0f0fu) | (((tmp >> 6) & 0x03030303u) << 4);
    uint32_t r0 = (a0 & 0x0f0f0f0fu) | (((tmp >> 0) & 0x03030303u) << 4);
    uint32_t r1 = (a1 & 0x0f0f0f0fu) | (((tmp >> 2) & 0x03030303u) << 4);
    const uint32_t aux[4] = {r0, r1, r2, r3};
    for (int i = 0; i < 16; i++) sc[i] = (int)(int8_t)(uint8_t)(aux[i / 4] >> (8 * (i % 4))) - 32;
}

// 2-bit code of weight w (0..255) of a Q2_K / Q3_K block's qs (bit planes)
static inline int q2_code(const uint8_t* q, int w) {
    int shift = 2 * ((w % 128) / 32);
    return (q[32 * (w / 128) + (w % 128) % 32] >> shift) & 3;
}

// EntropyCoder.Decode3 (EntropyCoder.cs:83-110): rANS, M = 256, L = 2^23.
// Returns -1 where the reference throws (truncated or corrupt stream).
static int rans_decode3(const uint8_t* src, int len, int n, uint32_t f0, uint32_t f1, uint8_t* out) {
    const uint32_t M = 256, L = 1u << 23;
    uint32_t f2 = M - f0 - f1;
    int p = 0;
    uint32_t x = 0;
    for (int b = 0; b < 4; b++) {
        if (p >= len) return -1;
        x = (x << 8) | src[p++];
    }
    for (int i = 0; i < n; i++) {
        while (x < L) {
            if (p >= len) return -1;
            x = (x << 8) | src[p++];
        }
        uint32_t slot = x & (M - 1), s, f, c;
        if (slot < f0) { s = 0; f = f0; c = 0; }
        else if (slot < f0 + f1) { s = 1; f = f1; c = f0; }
        else { s = 2; f = f2; c = f0 + f1; }
        if (f == 0) return -1;
        x = f * (x >> 8) + slot - c;
        out[i] = (uint8_t)s;
    }
    return 0;
}

int orc_dequantize(int fmt, const uint8_t* s, int64_t n, float* y) {
    int bs, bb;
    if (orc_block_spec(fmt, &bs, &bb) != 0 || n % bs != 0) return -1;
    int64_t nb = n / bs;
    switch (fmt) {
        case ORC_F32: std::memcpy(y, s, (size_t)n * 4); return 0;
        case ORC_F16: for (int64_t i = 0; i < n; i++) y[i] = orc_f16_to_f32(rd16(s + 2 * i)); return 0;
        case ORC_BF16: for (int64_t i = 0; i < n; i++) y[i] = orc_bf16_to_f32(rd16(s + 2 * i)); return 0;
        case ORC_Q4_0:  // BlockDequantizer.cs:52-69
            for (int64_t b = 0; b < nb; b++, s += 20, y += 32) {
                float d = orc_f16_to_f32(rd16(s));
                for (int i = 0; i < 16; i++) {
                    y[i] = d * ((s[2 + i] & 0xF) - 8);
                    y[i + 16] = d * ((s[2 + i] >> 4) - 8);
                }
            }
            return 0;
        case ORC_Q8_0:  // BlockDequantizer.cs:71-84
            for (int64_t b = 0; b < nb; b++, s += 34, y += 32) {
                float d = orc_f16_to_f32(rd16(s));
                for (int i = 0; i < 32; i++) y[i] = d * (int8_t)s[2 + i];
            }
            return 0;
        case ORC_Q4_K:  // BlockDequantizer.cs:168-195
            for (int64_t b = 0; b < nb; b++, s += 144, y += 256) {
                float d = orc_f16_to_f32(rd16(s));
                float dmin = orc_f16_to_f32(rd16(s + 2));
                const uint8_t* packed = s + 4;
                const uint8_t* q = s + 16;
                for (int sub = 0; sub < 8; sub++) {
                    int scI, mI;
                    scale_min_k4(sub, packed, &scI, &mI);
                    float a = d * scI, m = dmin * mI;
                    const uint8_t* qb = q + (sub / 2) * 32;
                    int wBase = sub * 32;
                    if ((sub & 1) == 0)
                        for (int i = 0; i < 32; i++) y[wBase + i] = a * (qb[i] & 0xF) - m;
                    else
                        for (int i = 0; i < 32; i++) y[wBase + i] = a * (qb[i] >> 4) - m;
                }
            }
            return 0;
        case ORC_Q6_K:  // BlockDequantizer.cs:228-256
            for (int64_t b = 0; b < nb; b++, s += 210, y += 256) {
                float d = orc_f16_to_f32(rd16(s + 208));
                const uint8_t* ql = s;
                const uint8_t* qh = s + 128;
                const uint8_t* sc = s + 192;
                for (int nn = 0; nn < 256; nn += 128) {
                    for (int l = 0; l < 32; l++) {
                        int isx = l / 16;
                        int q1 = (ql[nn / 2 + l] & 0xF) | (((qh[nn / 4 + l] >> 0) & 3) << 4);
                        int q2 = (ql[nn / 2 + l + 32] & 0xF) | (((qh[nn / 4 + l] >> 2) & 3) << 4);
                        int q3 = (ql[nn / 2 + l] >> 4) | (((qh[nn / 4 + l] >> 4) & 3) << 4);
                        int q4 = (ql[nn / 2 + l + 32] >> 4) | (((qh[nn / 4 + l] >> 6) & 3) << 4);
                        y[nn + l] = d * (int8_t)sc[8 * (nn / 128) + isx + 0] * (q1 - 32);
                        y[nn + l + 32] = d * (int8_t)sc[8 * (nn / 128) + isx + 2] * (q2 - 32);
                        y[nn + l + 64] = d * (int8_t)sc[8 * (nn / 128) + isx + 4] * (q3 - 32);
                        y[nn + l + 96] = d * (int8_t)sc[8 * (nn / 128) + isx + 6] * (q4 - 32);
                    }
                }
            }
            return 0;
        case ORC_TRI:  // BlockDequantizer.cs:258-276
            for (int64_t b = 0; b < nb; b++, s += 18, y += 64) {
                float scale = orc_f16_to_f32(rd16(s));
                for (int i = 0; i < 64; i++) {
                    int code = (s[2 + i / 4] >> (2 * (i & 3))) & 3;
                    y[i] = code == 1 ? scale : code == 2 ? -scale : 0.f;
                }
            }
            return 0;
        case ORC_Q2_K:  // BlockDequantizer.cs:87-114
            for (int64_t b = 0; b < nb; b++, s += 84, y += 256) {
                float d = orc_f16_to_f32(rd16(s + 80)), dmin = orc_f16_to_f32(rd16(s + 82));
                for (int sub = 0; sub < 16; sub++) {
                    float a = d * (s[sub] & 0xF), m = dmin * (s[sub] >> 4);
                    for (int i = 0; i < 16; i++) {
                        int w = sub * 16 + i;
                        y[w] = a * q2_code(s + 16, w) - m;
                    }
                }
            }
            return 0;
        case ORC_Q3_K:  // BlockDequantizer.cs:117-151
            for (int64_t b = 0; b < nb; b++, s += 110, y += 256) {
                float d = orc_f16_to_f32(rd16(s + 108));
                int sc[16];
                q3k_scales(s + 96, sc);
                for (int w = 0; w < 256; w++) {
                    int qv = q2_code(s + 32, w);
                    if ((s[w % 32] & (1 << (w / 32))) == 0) qv -= 4;
                    y[w] = d * sc[w / 16] * qv;
                }
            }
            return 0;
        case ORC_Q5_K:  // BlockDequantizer.cs:198-226
            for (int64_t b = 0; b < nb; b++, s += 176, y += 256) {
                float d = orc_f16_to_f32(rd16(s)), dmin = orc_f16_to_f32(rd16(s + 2));
                const uint8_t *packed = s + 4, *ql = s + 16, *qh = s + 144;
                for (int sub = 0; sub < 8; sub++) {
                    int scI, mI;
                    scale_min_k4(sub, packed, &scI, &mI);
                    float a = d * scI, m = dmin * mI;
                    int j = sub / 2;
                    const uint8_t* q = ql + j * 32;
                    int u1 = 1 << (2 * j), u2 = 2 << (2 * j);
                    if ((sub & 1) == 0)
                        for (int i = 0; i < 32; i++) y[sub * 32 + i] = a * ((q[i] & 0xF) + ((qh[i] & u1) != 0 ? 16 : 0)) - m;
                    else
                        for (int i = 0; i < 32; i++) y[sub * 32 + i] = a * ((q[i] >> 4) + ((qh[i] & u2) != 0 ? 16 : 0)) - m;
                }
            }
            return 0;
        case ORC_I8_BLK:  // BlockDequantizer.cs:278-290
            for (int64_t b = 0; b < nb; b++, s += 258, y += 256) {
                float d = orc_f16_to_f32(rd16(s));
                for (int i = 0; i < 256; i++) y[i] = d * (int8_t)s[2 + i];
            }
            return 0;
        case ORC_B1:  // BlockDequantizer.cs:299-313
        case ORC_B1X:  // BlockDequantizer.cs:315-336
            for (int64_t b = 0; b < nb; b++, s += bb, y += 256) {
                float a = orc_f16_to_f32(rd16(s));
                for (int i = 0; i < 256; i++) y[i] = (s[2 + (i >> 3)] & (1 << (i & 7))) != 0 ? a : -a;
                if (fmt == ORC_B1X) {
                    int k = s[34];
                    for (int e = 0; e < k; e++) y[s[35 + 3 * e]] = orc_f16_to_f32(rd16(s + 35 + 3 * e + 1));
                }
            }
            return 0;
        case ORC_T1E:  // BlockDequantizer.cs:338-359
        case ORC_T1E_LO:
            for (int64_t b = 0; b < nb; b++, s += bb, y += 256) {
                uint8_t syms[256];
                float a = orc_f16_to_f32(rd16(s + 4));
                if (rans_decode3(s + 6, bb - 6, 256, rd16(s), rd16(s + 2), syms) != 0) return -1;
                for (int i = 0; i < 256; i++) y[i] = syms[i] == 1 ? a : syms[i] == 2 ? -a : 0.f;
            }
            return 0;
        default: return -1;
    }
}

// ------------------------------------------------------------ DotKernels.cs

// SimdMath.HSum(Vector256<float>), SimdMath.cs:17-22: sequential lane sum.
static inline float hsum8(const float* acc) {
    float s = 0;
    for (int i = 0; i < 8; i++) s += acc[i];
    return s;
}

float orc_dot_f32(const float* a, const float* b, int n) {
    // SimdMath.DotF32, SimdMath.cs:34-53 (Vector256 path for n >= 8)
    if (n >= 8) {
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        int i = 0;
        for (; i + 8 <= n; i += 8)
            for (int j = 0; j < 8; j++) acc[j] = acc[j] + a[i + j] * b[i + j];
        float s = hsum8(acc);
        for (; i < n; i++) s += a[i] * b[i];
        return s;
    }
    float ss = 0;
    for (int i = 0; i < n; i++) ss += a[i] * b[i];
    return ss;
}

static float dot_f16(const uint8_t* w, const float* x, int cols, bool bf16) {
    // DotKernels.DotF16 / DotBf16 (DotKernels.cs:57-128): exact widening then
    // the same 8-lane accumulation as DotF32.
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int i = 0;
    auto cvt = [&](int k) { uint16_t h = rd16(w + 2 * k); return bf16 ? orc_bf16_to_f32(h) : orc_f16_to_f32(h); };
    if (cols >= 8) {
        for (; i + 8 <= cols; i += 8)
            for (int j = 0; j < 8; j++) acc[j] = acc[j] + cvt(i + j) * x[i + j];
        float sum = hsum8(acc);
        for (; i < cols; i++) sum += cvt(i) * x[i];
        return sum;
    }
    float ss = 0;
    for (int k = 0; k < cols; k++) ss += cvt(k) * x[k];
    return ss;
}

static float dot_q4_0(const uint8_t* w, const float* x, int cols) {
    // DotKernels.DotQ4_0, DotKernels.cs:132-179 (Vector256 branch)
    int nb = cols / 32;
    float sum = 0.f;
    for (int b = 0; b < nb; b++, w += 20, x += 32) {
        float d = orc_f16_to_f32(rd16(w));
        float lo[16], hi[16];
        for (int i = 0; i < 16; i++) { lo[i] = (float)(w[2 + i] & 0xF); hi[i] = (float)(w[2 + i] >> 4); }
        float accQ[8] = {0, 0, 0, 0, 0, 0, 0, 0}, accX[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int j = 0; j < 8; j++) accQ[j] = accQ[j] + lo[j] * x[j];
        for (int j = 0; j < 8; j++) accQ[j] = accQ[j] + lo[8 + j] * x[8 + j];
        for (int j = 0; j < 8; j++) accQ[j] = accQ[j] + hi[j] * x[16 + j];
        for (int j = 0; j < 8; j++) accQ[j] = accQ[j] + hi[8 + j] * x[24 + j];
        for (int j = 0; j < 8; j++) accX[j] = accX[j] + x[j];
        for (int j = 0; j < 8; j++) accX[j] = accX[j] + x[8 + j];
        for (int j = 0; j < 8; j++) accX[j] = accX[j] + x[16 + j];
        for (int j = 0; j < 8; j++) accX[j] = accX[j] + x[24 + j];
        float dotQ = hsum8(accQ);
        float sumX = hsum8(accX);
        sum += d * dotQ - 8.f * d * sumX;
    }
    return sum;
}

static float dot_q8_0(const uint8_t* w, const float* x, int cols) {
    // DotKernels.DotQ8_0 + DotI8Bytes, DotKernels.cs:184-235 (Vector256 branch)
    int nb = cols / 32;
    float sum = 0.f;
    for (int b = 0; b < nb; b++, w += 34, x += 32) {
        float d = orc_f16_to_f32(rd16(w));
        const uint8_t* q = w + 2;
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int i = 0; i + 16 <= 32; i += 16) {
            for (int j = 0; j < 8; j++) acc[j] = acc[j] + (float)(int8_t)q[i + j] * x[i + j];
            for (int j = 0; j < 8; j++) acc[j] = acc[j] + (float)(int8_t)q[i + 8 + j] * x[i + 8 + j];
        }
        float dot = hsum8(acc);
        sum += d * dot;
    }
    return sum;
}

// DotKernels.VecDot16, DotKernels.cs:360-373 (vector branch)
static inline float vecdot16(const float* q, const float* x) {
    float acc[8];
    for (int j = 0; j < 8; j++) acc[j] = q[j] * x[j];
    for (int j = 0; j < 8; j++) acc[j] = acc[j] + q[8 + j] * x[8 + j];
    return hsum8(acc);
}

// DotKernels.SubSum, DotKernels.cs:270-275
static inline float subsum(const float* x, int n) {
    float s = 0;
    for (int i = 0; i < n; i++) s += x[i];
    return s;
}

static float dot_q4_k(const uint8_t* w, const float* x, int cols) {
    // DotKernels.DotQ4_K, DotKernels.cs:325-357 (vector branch)
    int nb = cols / 256;
    float sum = 0.f;
    float lo[16], hi[16];
    for (int b = 0; b < nb; b++, w += 144, x += 256) {
        float d = orc_f16_to_f32(rd16(w));
        float dmin = orc_f16_to_f32(rd16(w + 2));
        const uint8_t* packed = w + 4;
        const uint8_t* q = w + 16;
        for (int j = 0; j < 4; j++, q += 32) {
            int sc0, m0, sc1, m1;
            scale_min_k4(2 * j, packed, &sc0, &m0);
            float a0 = d * sc0, mm0 = dmin * m0;
            for (int i = 0; i < 16; i++) { lo[i] = (float)(q[i] & 0xF); hi[i] = (float)(q[16 + i] & 0xF); }
            {
                float t1 = vecdot16(lo, x + j * 64);
                float t2 = vecdot16(hi, x + j * 64 + 16);
                float ss = subsum(x + j * 64, 32);
                sum += a0 * (t1 + t2) - mm0 * ss;
            }
            scale_min_k4(2 * j + 1, packed, &sc1, &m1);
            float a1 = d * sc1, mm1 = dmin * m1;
            for (int i = 0; i < 16; i++) { lo[i] = (float)(q[i] >> 4); hi[i] = (float)(q[16 + i] >> 4); }
            {
                float t1 = vecdot16(lo, x + j * 64 + 32);
                float t2 = vecdot16(hi, x + j * 64 + 48);
                float ss = subsum(x + j * 64 + 32, 32);
                sum += a1 * (t1 + t2) - mm1 * ss;
            }
        }
    }
    return sum;
}

static float dot_q6_k(const uint8_t* w, const float* x, int cols) {
    // DotKernels.DotQ6_K, DotKernels.cs:423-451: integer sc*(q-32), then
    // one float multiply and one float add per weight.
    int nb = cols / 256;
    float sum = 0.f;
    for (int b = 0; b < nb; b++, w += 210, x += 256) {
        float d = orc_f16_to_f32(rd16(w + 208));
        const uint8_t* ql = w;
        const uint8_t* qh = w + 128;
        const uint8_t* sc = w + 192;
        float dot = 0;
        for (int nn = 0; nn < 256; nn += 128) {
            int scBase = 8 * (nn / 128);
            for (int l = 0; l < 32; l++) {
                int isx = l / 16;
                int q1 = (ql[nn / 2 + l] & 0xF) | (((qh[nn / 4 + l] >> 0) & 3) << 4);
                int q2 = (ql[nn / 2 + l + 32] & 0xF) | (((qh[nn / 4 + l] >> 2) & 3) << 4);
                int q3 = (ql[nn / 2 + l] >> 4) | (((qh[nn / 4 + l] >> 4) & 3) << 4);
                int q4 = (ql[nn / 2 + l + 32] >> 4) | (((qh[nn / 4 + l] >> 6) & 3) << 4);
                dot += (float)((int8_t)sc[scBase + isx + 0] * (q1 - 32)) * x[nn + l];
                dot += (float)((int8_t)sc[scBase + isx + 2] * (q2 - 32)) * x[nn + l + 32];
                dot += (float)((int8_t)sc[scBase + isx + 4] * (q3 - 32)) * x[nn + l + 64];
                dot += (float)((int8_t)sc[scBase + isx + 6] * (q4 - 32)) * x[nn + l + 96];
            }
        }
        sum += d * dot;
    }
    return sum;
}

static float dot_tri(const uint8_t* w, const float* x, int cols) {
    // DotKernels.DotTri, DotKernels.cs:456-471 + SimdMath.UnpackTri 187-198
    int nb = cols / 64;
    float sum = 0.f;
    float qf[64];
    for (int b = 0; b < nb; b++, w += 18, x += 64) {
        float scale = orc_f16_to_f32(rd16(w));
        for (int i = 0; i < 16; i++) {
            uint8_t v = w[2 + i];
            for (int c = 0; c < 4; c++) {
                int code = (v >> (2 * c)) & 3;
                qf[4 * i + c] = code == 1 ? scale : code == 2 ? -scale : 0.f;
            }
        }
        float dot = 0;
        for (int i = 0; i < 64; i++) dot += qf[i] * x[i];
        sum += dot;
    }
    return sum;
}

static float dot_q2_k(const uint8_t* w, const float* x, int cols) {
    // DotKernels.DotQ2_K, DotKernels.cs:240-266 (+ SubSum 270-275)
    int nb = cols / 256;
    float sum = 0.f;
    for (int b = 0; b < nb; b++, w += 84, x += 256) {
        float d = orc_f16_to_f32(rd16(w + 80)), dmin = orc_f16_to_f32(rd16(w + 82));
        for (int sub = 0; sub < 16; sub++) {
            float a = d * (w[sub] & 0xF);
            float m = dmin * (w[sub] >> 4);
            int r = sub * 16;
            float dsub = 0;
            for (int i = 0; i < 16; i++) dsub += q2_code(w + 16, r + i) * x[r + i];
            sum += a * dsub - m * subsum(x + r, 16);
        }
    }
    return sum;
}

static float dot_q3_k(const uint8_t* w, const float* x, int cols) {
    // DotKernels.DotQ3_K, DotKernels.cs:280-318
    int nb = cols / 256;
    float sum = 0.f;
    int sc[16];
    for (int b = 0; b < nb; b++, w += 110, x += 256) {
        float d = orc_f16_to_f32(rd16(w + 108));
        q3k_scales(w + 96, sc);
        for (int sub = 0; sub < 16; sub++) {
            float a = d * sc[sub];
            int r = sub * 16;
            float dsub = 0;
            for (int i = 0; i < 16; i++) {
                int wI = r + i;
                int qv = q2_code(w + 32, wI);
                if ((w[wI % 32] & (1 << (wI / 32))) == 0) qv -= 4;
                dsub += qv * x[wI];
            }
            sum += a * dsub;
        }
    }
    return sum;
}

static float dot_q5_k(const uint8_t* w, const float* x, int cols) {
    // DotKernels.DotQ5_K, DotKernels.cs:378-418
    int nb = cols / 256;
    float sum = 0.f;
    for (int b = 0; b < nb; b++, w += 176, x += 256) {
        float d = orc_f16_to_f32(rd16(w)), dmin = orc_f16_to_f32(rd16(w + 2));
        const uint8_t *packed = w + 4, *ql = w + 16, *qh = w + 144;
        for (int sub = 0; sub < 8; sub++) {
            int scI, mI;
            scale_min_k4(sub, packed, &scI, &mI);
            float a = d * scI, m = dmin * mI;
            int j = sub / 2;
            const uint8_t* q = ql + j * 32;
            int u1 = 1 << (2 * j), u2 = 2 << (2 * j);
            float dsub = 0, xsub = 0;
            int wBase = sub * 32;
            for (int i = 0; i < 32; i++) {
                int q5 = (sub & 1) == 0 ? (q[i] & 0xF) + ((qh[i] & u1) != 0 ? 16 : 0)
                                        : (q[i] >> 4) + ((qh[i] & u2) != 0 ? 16 : 0);
                dsub += q5 * x[wBase + i];
                xsub += x[wBase + i];
            }
            sum += a * dsub - m * xsub;
        }
    }
    return sum;
}

// DotKernels.DotI8Bytes (vector branch), DotKernels.cs:209-234, n = 16:
// two 8-lane products added into one accumulator, then HSum
static float dot_i8_bytes16(const uint8_t* q, const float* x) {
    float acc[8];
    for (int l = 0; l < 8; l++) acc[l] = 0.f + (float)(int8_t)q[l] * x[l];
    for (int l = 0; l < 8; l++) acc[l] = acc[l] + (float)(int8_t)q[8 + l] * x[8 + l];
    return hsum8(acc);
}

static float dot_i8_blk(const uint8_t* w, const float* x, int cols) {
    // DotKernels.DotI8Blk, DotKernels.cs:476-495 (vector branch)
    int nb = cols / 256;
    float sum = 0.f;
    for (int b = 0; b < nb; b++, w += 258, x += 256) {
        float d = orc_f16_to_f32(rd16(w));
        float dot = 0;
        for (int i = 0; i < 256; i += 16) dot += dot_i8_bytes16(w + 2 + i, x + i);
        sum += d * dot;
    }
    return sum;
}

static float dot_b1(const uint8_t* w, const float* x, int cols, bool exc) {
    // DotKernels.DotB1 / DotB1X (DotKernels.cs:515-556) with ExpandSigns 559-569
    int nb = cols / 256, bb = exc ? 47 : 34;
    float sum = 0.f;
    float sf[256];
    for (int b = 0; b < nb; b++, w += bb, x += 256) {
        float a = orc_f16_to_f32(rd16(w));
        for (int i = 0; i < 256; i++) sf[i] = (w[2 + (i >> 3)] & (1 << (i & 7))) != 0 ? 1.f : -1.f;
        sum += a * orc_dot_f32(sf, x, 256);
        if (exc) {
            int k = w[34];
            for (int e = 0; e < k; e++) {
                int idx = w[35 + 3 * e];
                float v = orc_f16_to_f32(rd16(w + 35 + 3 * e + 1));
                float sgn = (w[2 + (idx >> 3)] & (1 << (idx & 7))) != 0 ? 1.f : -1.f;
                sum += (v - a * sgn) * x[idx];
            }
        }
    }
    return sum;
}

static float dot_t1e(const uint8_t* w, const float* x, int cols, int stream) {
    // DotKernels.DotT1E, DotKernels.cs:572-593
    int nb = cols / 256;
    float sum = 0.f;
    uint8_t syms[256];
    for (int b = 0; b < nb; b++, w += 6 + stream, x += 256) {
        float a = orc_f16_to_f32(rd16(w + 4));
        if (rans_decode3(w + 6, stream, 256, rd16(w), rd16(w + 2), syms) != 0) return NAN;
        float dot = 0;
        for (int i = 0; i < 256; i++) {
            float v = syms[i] == 1 ? a : syms[i] == 2 ? -a : 0.f;
            dot += v * x[i];
        }
        sum += dot;
    }
    return sum;
}

float orc_dot_row(int fmt, const uint8_t* w, const float* x, int cols) {
    switch (fmt) {
        case ORC_F32: {
            std::vector<float> a((size_t)cols);
            std::memcpy(a.data(), w, (size_t)cols * 4);
            return orc_dot_f32(a.data(), x, cols);
        }
        case ORC_F16: return dot_f16(w, x, cols, false);
        case ORC_BF16: return dot_f16(w, x, cols, true);
        case ORC_Q4_0: return dot_q4_0(w, x, cols);
        case ORC_Q8_0: return dot_q8_0(w, x, cols);
        case ORC_Q4_K: return dot_q4_k(w, x, cols);
        case ORC_Q6_K: return dot_q6_k(w, x, cols);
        case ORC_TRI: return dot_tri(w, x, cols);
        case ORC_Q2_K: return dot_q2_k(w, x, cols);
        case ORC_Q3_K: return dot_q3_k(w, x, cols);
        case ORC_Q5_K: return dot_q5_k(w, x, cols);
        case ORC_I8_BLK: return dot_i8_blk(w, x, cols);
        case ORC_B1: return dot_b1(w, x, cols, false);
        case ORC_B1X: return dot_b1(w, x, cols, true);
        case ORC_T1E: return dot_t1e(w, x, cols, 34);
        case ORC_T1E_LO: return dot_t1e(w, x, cols, 26);
        default: return NAN;
    }
}

static int64_t row_bytes(int fmt, int64_t cols) {
    int bs, bb;
    if (orc_block_spec(fmt, &bs, &bb) != 0) return -1;
    return cols / bs * bb;
}

int orc_matvec(int fmt, const uint8_t* w, int64_t rows, int64_t cols, const float* x, float* y) {
    // DotKernels.MatVec, DotKernels.cs:599-607
    int64_t rb = row_bytes(fmt, cols);
    if (rb < 0) return -1;
    if (fmt == ORC_F32) {
        for (int64_t r = 0; r < rows; r++) y[r] = orc_dot_f32((const float*)(w + r * rb), x, (int)cols);
        return 0;
    }
    for (int64_t r = 0; r < rows; r++) y[r] = orc_dot_row(fmt, w + r * rb, x, (int)cols);
    return 0;
}

int orc_matvec_parallel(int fmt, const uint8_t* w, int64_t rows, int64_t cols, const float* x,
                        float* y, int threads) {
    // DotKernels.MatVecParallel, DotKernels.cs:610-629 (minRowsPerThread = 8)
    int64_t rb = row_bytes(fmt, cols);
    if (rb < 0) return -1;
    if (threads < 1) threads = 1;
    if (threads == 1 || rows < 8 * 2 || rows * rb < (1 << 20)) return orc_matvec(fmt, w, rows, cols, x, y);
    int64_t chunk = (rows + threads - 1) / threads;
    std::vector<std::thread> pool;
    pool.reserve((size_t)threads);
    for (int t = 0; t < threads; t++) {
        int64_t r0 = t * chunk, r1 = std::min(rows, r0 + chunk);
        if (r0 >= r1) break;
        pool.emplace_back([=]() { orc_matvec(fmt, w + r0 * rb, r1 - r0, cols, x, y + r0); });
    }
    for (auto& th : pool) th.join();
    return 0;
}

// ------------------------------------------------------- TransformerOps.cs

void orc_rmsnorm(const float* x, const float* w, float* out, int n, float eps) {
    // TransformerOps.RmsNorm, TransformerOps.cs:12-40
    float ss = 0;
    int i = 0;
    if (n >= 8) {
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (; i + 8 <= n; i += 8)
            for (int j = 0; j < 8; j++) acc[j] = acc[j] + x[i + j] * x[i + j];
        ss = hsum8(acc);
    }
    for (; i < n; i++) ss += x[i] * x[i];
    float scale = 1.f / std::sqrt(ss / (float)n + eps);
    for (i = 0; i < n; i++) out[i] = x[i] * scale;
    if (w != nullptr)
        for (i = 0; i < n; i++) out[i] *= w[i];
}

void orc_expf_batch(const float* x, float* y, int64_t n) {
    for (int64_t i = 0; i < n; i++) y[i] = expf(x[i]);
}

void orc_swiglu(float* g, const float* u, int n, float limit) {
    if (limit <= 0) {
        // TransformerOps.SiluMulInPlace, TransformerOps.cs:114-121
        for (int i = 0; i < n; i++) {
            float gv = g[i];
            g[i] = gv / (1.f + expf(-gv)) * u[i];
        }
        return;
    }
    // Glm5Ops.LimitedSwiglu, Glm5Ops.cs:243-256 (Silu = v / (1 + exp(-v)))
    for (int i = 0; i < n; i++) {
        float gv = g[i] > limit ? limit : g[i];
        float uv = u[i];
        uv = uv > limit ? limit : (uv < -limit ? -limit : uv);
        g[i] = gv / (1.f + expf(-gv)) * uv;
    }
}

// ------------------------------------------------------ routing (StreamingEngine)

// Sort order of Array.Sort(idx, (a, b) => v[b].CompareTo(v[a])): descending,
// NaN last (float.CompareTo orders NaN lowest).  Exact ties: index ascending.
static inline bool ranks_before(float va, int ia, float vb, int ib) {
    bool na = std::isnan(va), nb = std::isnan(vb);
    if (na != nb) return nb;
    if (!na && va != vb) return va > vb;
    return ia < ib;
}

static void topk_order(const float* v, int n, int k, int* out) {
    std::vector<int> idx((size_t)n);
    for (int i = 0; i < n; i++) idx[(size_t)i] = i;
    int kk = std::min(k, n);
    std::partial_sort(idx.begin(), idx.begin() + kk, idx.end(),
                      [&](int a, int b) { return ranks_before(v[a], a, v[b], b); });
    for (int i = 0; i < kk; i++) out[i] = idx[(size_t)i];
}

void orc_route_softmax(const float* logits, int E, int k, int32_t* sel, float* wsel, float* probs) {
    // MoeFfn routing, StreamingEngine.cs:642-652 + SelectTopK 801-810
    std::vector<float> p(logits, logits + E);
    float max = -3.40282347e+38f;  // float.MinValue
    for (int i = 0; i < E; i++) if (p[(size_t)i] > max) max = p[(size_t)i];
    float sum = 0;
    for (int i = 0; i < E; i++) { p[(size_t)i] = expf(p[(size_t)i] - max); sum += p[(size_t)i]; }
    float inv = 1.f / sum;
    for (int i = 0; i < E; i++) p[(size_t)i] *= inv;
    int idx[8];
    topk_order(p.data(), E, k, idx);
    float s = 0;
    for (int i = 0; i < k; i++) s += p[(size_t)idx[i]];
    if (s <= 0) s = 1;
    for (int i = 0; i < k; i++) { sel[i] = idx[i]; wsel[i] = p[(size_t)idx[i]] / s; }
    if (probs) std::memcpy(probs, p.data(), sizeof(float) * (size_t)E);
}

void orc_route_sigmoid(const float* logits, const float* bias, int E, int k, float routed_scale,
                       int32_t* sel, float* wsel) {
    // GlmMoeFfn routing, StreamingEngine.cs:730-767; Glm5Ops.Sigmoid, Glm5Ops.cs:19
    int nExp = std::min(E, 512);
    std::vector<float> scores((size_t)nExp), choice((size_t)nExp);
    for (int i = 0; i < nExp; i++) {
        scores[(size_t)i] = 1.f / (1.f + expf(-logits[i]));
        choice[(size_t)i] = bias ? scores[(size_t)i] + bias[i] : scores[(size_t)i];
    }
    int idx[8];
    topk_order(choice.data(), nExp, k, idx);
    float wsum = 0;
    for (int e = 0; e < k; e++) wsum += scores[(size_t)idx[e]];
    float inv2 = 1.f / (wsum + 1e-20f);
    for (int e = 0; e < k; e++) {
        sel[e] = idx[e];
        wsel[e] = scores[(size_t)idx[e]] * inv2 * routed_scale;
    }
}

void orc_dispatch(const int32_t* sel, int T, int k, int E, int32_t* perm, int32_t* inv_perm,
                  int32_t* offsets) {
    std::vector<int32_t> cnt((size_t)E + 1, 0);
    int n = T * k;
    for (int a = 0; a < n; a++) cnt[(size_t)sel[a] + 1]++;
    for (int e = 0; e < E; e++) cnt[(size_t)e + 1] += cnt[(size_t)e];
    if (offsets) std::memcpy(offsets, cnt.data(), sizeof(int32_t) * ((size_t)E + 1));
    for (int a = 0; a < n; a++) {
        int pos = cnt[(size_t)sel[a]]++;
        if (perm) perm[pos] = a;
        if (inv_perm) inv_perm[a] = pos;
    }
}

// ------------------------------------------------------------ MoE layer

// RMSNorm, router logits (+ harness offset) and top-k of one token: the part
// of MoeFfn / GlmMoeFfn before the experts (StreamingEngine.cs:259-260,
// 639-652, 727-767).
static void route_token(const orc_moe_desc* desc, const orc_moe_weights* w, const float* xt, int flags, int k,
                        float* xn, float* logits, int32_t* sel, float* wsel, int threads) {
    const int d = desc->d_model, E = desc->n_experts;
    if (flags & ORC_APPLY_NORM) orc_rmsnorm(xt, w->norm_w, xn, d, desc->rms_eps);
    else std::memcpy(xn, xt, sizeof(float) * (size_t)d);
    // router logits: MatVecParallel(F32) over the [E x d] router
    orc_matvec_parallel(ORC_F32, (const uint8_t*)w->router, E, d, xn, logits, threads);
    if (w->logit_offset)
        for (int e = 0; e < E; e++) logits[e] = logits[e] + w->logit_offset[e];
    if (desc->moe_sigmoid)
        orc_route_sigmoid(logits, w->router_bias, E, k, desc->routed_scale, sel, wsel);
    else
        orc_route_softmax(logits, E, k, sel, wsel, nullptr);
}

int orc_moe_route(const orc_moe_desc* desc, const orc_moe_weights* w, const float* x, int T, int flags,
                  int32_t* topk_idx, float* topk_w, float* logits_out, float* xn_out, int threads) {
    const int d = desc->d_model, E = desc->n_experts;
    const int k = std::min(desc->n_active, 8);
    if (d <= 0 || E <= 0 || k <= 0 || k > E) return -1;
    std::vector<float> xn((size_t)d), logits((size_t)E);
    for (int t = 0; t < T; t++) {
        int32_t sel[8];
        float wsel[8];
        route_token(desc, w, x + (size_t)t * d, flags, k, xn.data(), logits.data(), sel, wsel, threads);
        if (xn_out) std::memcpy(xn_out + (size_t)t * d, xn.data(), sizeof(float) * (size_t)d);
        if (logits_out) std::memcpy(logits_out + (size_t)t * E, logits.data(), sizeof(float) * (size_t)E);
        if (topk_idx) std::memcpy(topk_idx + (size_t)t * k, sel, sizeof(int32_t) * (size_t)k);
        if (topk_w) std::memcpy(topk_w + (size_t)t * k, wsel, sizeof(float) * (size_t)k);
    }
    return 0;
}

int orc_moe_forward(const orc_moe_desc* desc, const orc_moe_weights* w, const float* x, int T,
                    int flags, float* out, int32_t* topk_idx, float* topk_w, float* logits_out,
                    float* xn_out, int threads) {
    const int d = desc->d_model, E = desc->n_experts, f = desc->expert_ffn;
    const int k = std::min(desc->n_active, 8);
    if (d <= 0 || E <= 0 || f <= 0 || k <= 0 || k > E) return -1;
    std::vector<float> xn((size_t)d), logits((size_t)E), g((size_t)f), u((size_t)f), y((size_t)d);
    for (int t = 0; t < T; t++) {
        const float* xt = x + (size_t)t * d;
        float* ot = out + (size_t)t * d;
        int32_t sel[8];
        float wsel[8];
        route_token(desc, w, xt, flags, k, xn.data(), logits.data(), sel, wsel, threads);
        if (xn_out) std::memcpy(xn_out + (size_t)t * d, xn.data(), sizeof(float) * (size_t)d);
        if (logits_out) std::memcpy(logits_out + (size_t)t * E, logits.data(), sizeof(float) * (size_t)E);
        if (topk_idx) std::memcpy(topk_idx + (size_t)t * k, sel, sizeof(int32_t) * (size_t)k);
        if (topk_w) std::memcpy(topk_w + (size_t)t * k, wsel, sizeof(float) * (size_t)k);
        // MoeFfn accumulates into the residual x; the other two start from 0.
        if (flags & ORC_ADD_RESIDUAL) std::memcpy(ot, xt, sizeof(float) * (size_t)d);
        else for (int i = 0; i < d; i++) ot[i] = 0;
        float limit = desc->moe_sigmoid ? desc->swiglu_limit : 0.f;
        for (int j = 0; j < k; j++) {
            int e = sel[j];
            orc_matvec_parallel(w->fmt_gate, w->gate[e], f, d, xn.data(), g.data(), threads);
            orc_matvec_parallel(w->fmt_up, w->up[e], f, d, xn.data(), u.data(), threads);
            orc_swiglu(g.data(), u.data(), f, limit);
            orc_matvec_parallel(w->fmt_down, w->down[e], d, f, g.data(), y.data(), threads);
            // SimdMath.AxpyF32 (SimdMath.cs:55-71): out = out + w * y
            float wj = wsel[j];
            for (int i = 0; i < d; i++) ot[i] = ot[i] + wj * y[(size_t)i];
        }
        if (desc->moe_sigmoid && desc->n_shared > 0 && w->sh_gate) {
            // StreamingEngine.cs:779-789: shared expert, weight 1
            orc_matvec_parallel(w->fmt_sh_gate, w->sh_gate, f, d, xn.data(), g.data(), threads);
            orc_matvec_parallel(w->fmt_sh_up, w->sh_up, f, d, xn.data(), u.data(), threads);
            orc_swiglu(g.data(), u.data(), f, limit);
            orc_matvec_parallel(w->fmt_sh_down, w->sh_down, d, f, g.data(), y.data(), threads);
            for (int i = 0; i < d; i++) ot[i] = ot[i] + 1.f * y[(size_t)i];
        }
    }
    return 0;
}

}  // extern "C"
