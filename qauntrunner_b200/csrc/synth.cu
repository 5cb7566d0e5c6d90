// synth.cu -- synthetic expert weights on the device: a counter-based
// Gaussian generator and the reference quantisers (BlockQuantizer.cs), one
// thread per block.  This is the device counterpart of the reference's
// `synthesize` command (src/QuantRunner.Cli/Program.cs:247-369), used to make
// the large benchmark layers without a CPU round trip; the forward path never
// quantises.  Compiled with -fmad=false: every float expression below is the
// same sequence of binary32/binary64 operations as the C# quantiser, so the
// bytes equal the CPU quantiser's (checked by tests/test_gpu_synth.py).
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/qrmoe.h"
#include "common.cuh"

namespace qrm {

__device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// N(0,1) by Box-Muller sqrt(-2 ln(1-u1)) * sin(2 pi u2), as NextGaussian
// (Program.cs:373-377), with u1, u2 from splitmix64 of (seed, index).
__global__ void gaussian_kernel(float* __restrict__ dst, long long n, uint64_t seed, float sigma) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        uint64_t a = splitmix64(seed * 0x632BE59BD9B4E019ull + 2ull * (uint64_t)i);
        uint64_t b = splitmix64(seed * 0x632BE59BD9B4E019ull + 2ull * (uint64_t)i + 1ull);
        double u1 = 1.0 - (double)(a >> 11) * (1.0 / 9007199254740992.0);  // (0, 1]
        double u2 = (double)(b >> 11) * (1.0 / 9007199254740992.0);
        double g = sqrt(-2.0 * log(u1)) * sin(2.0 * 3.141592653589793 * u2);
        dst[i] = (float)g * sigma;
    }
}

// ------------------------------------------------ Dtypes.FloatToF16 (Dtypes.cs:100-126)
__device__ uint16_t f32_to_f16_ref(float f) {
    uint32_t x = __float_as_uint(f);
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

// C# (int)MathF.Round(v): ties-to-even, then truncation (x64: INT_MIN when out of range)
__device__ __forceinline__ int round_int(float v) {
    float r = rintf(v);
    if (!(r > -2147483904.0f && r < 2147483648.0f)) return INT32_MIN;
    return (int)r;
}
__device__ __forceinline__ int clampq(int v, int lo, int hi) { return v < lo ? lo : v > hi ? hi : v; }
__device__ __forceinline__ void put16(uint8_t* p, uint16_t v) { p[0] = (uint8_t)(v & 0xFF); p[1] = (uint8_t)(v >> 8); }

__device__ void q4_0_block(const float* x, uint8_t* y) {  // BlockQuantizer.cs:69-93
    float amax = 0.f;
    for (int i = 0; i < 32; i++) { float a = fabsf(x[i]); if (a > amax) amax = a; }
    float d = amax / 8.f;
    put16(y, f32_to_f16_ref(d));
    y[18] = 0; y[19] = 0;
    if (d == 0.f) { for (int i = 0; i < 16; i++) y[2 + i] = 8; return; }
    float id = 1.f / d;
    for (int i = 0; i < 16; i++) {
        int q0 = clampq(round_int(x[i] * id) + 8, 0, 15);
        int q1 = clampq(round_int(x[i + 16] * id) + 8, 0, 15);
        y[2 + i] = (uint8_t)(q0 | (q1 << 4));
    }
}

__device__ void q8_0_block(const float* x, uint8_t* y) {  // BlockQuantizer.cs:97-116
    float amax = 0.f;
    for (int i = 0; i < 32; i++) { float a = fabsf(x[i]); if (a > amax) amax = a; }
    float d = amax / 127.f;
    put16(y, f32_to_f16_ref(d));
    if (d == 0.f) { for (int i = 0; i < 32; i++) y[2 + i] = 0; return; }
    float id = 1.f / d;
    for (int i = 0; i < 32; i++) y[2 + i] = (uint8_t)(int8_t)clampq(round_int(x[i] * id), -128, 127);
}

// BlockQuantizer.cs:248-318.  `L` is the code buffer; a sub-block whose scale
// rounds to 0 keeps whatever `L` held (see quantize_kernel).
__device__ void q4_k_block(const float* x, uint8_t* y, uint8_t* L) {
    float mins[8], maxs[8];
    int sc[8], m[8];
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
    for (int i = 0; i < 144; i++) y[i] = 0;
    if (amax <= 0.f) return;
    float d = amax / 945.f, dmin = amink > 0 ? amink / 63.f : 0.f;
    put16(y, f32_to_f16_ref(d));
    put16(y + 2, f32_to_f16_ref(dmin));
    float iscale = 63.f / amax, ismin = dmin > 0 ? 63.f / amink : 0.f;
    for (int s = 0; s < 8; s++) {
        sc[s] = clampq(round_int(iscale * (maxs[s] - mins[s])), 0, 63);
        m[s] = dmin > 0 ? clampq(round_int(ismin * (-mins[s])), 0, 63) : 0;
    }
    for (int j = 0; j < 4; j++) {
        y[4 + j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
        y[4 + j + 4] = (uint8_t)((m[j] & 63) | ((m[j + 4] >> 4) << 6));
        y[4 + j + 8] = (uint8_t)((sc[j + 4] & 0xF) | ((m[j + 4] & 0xF) << 4));
    }
    for (int s = 0; s < 8; s++) {
        float a = d * sc[s], bias = dmin * m[s];
        if (a <= 0.f) continue;
        for (int i = 0; i < 32; i++) L[s * 32 + i] = (uint8_t)clampq(round_int((x[s * 32 + i] + bias) / a), 0, 15);
    }
    for (int s = 0; s < 8; s++) {
        int baseByte = 16 + (s / 2) * 32;
        for (int i = 0; i < 32; i++) {
            int val = L[s * 32 + i];
            if ((s & 1) == 0) y[baseByte + i] |= (uint8_t)val;
            else y[baseByte + i] |= (uint8_t)(val << 4);
        }
    }
}

__device__ void q6_k_block(const float* x, uint8_t* y) {  // BlockQuantizer.cs:398-446
    float subAmax[16];
    int sc[16];
    float amax = 0.f;
    for (int s = 0; s < 16; s++) {
        float mx = 0.f;
        for (int i = 0; i < 16; i++) { float a = fabsf(x[s * 16 + i]); if (a > mx) mx = a; }
        subAmax[s] = mx;
        if (mx > amax) amax = mx;
    }
    for (int i = 0; i < 210; i++) y[i] = 0;
    if (amax <= 0.f) return;
    float d = amax / (31.f * 31.f);
    put16(y + 208, f32_to_f16_ref(d));
    for (int s = 0; s < 16; s++) sc[s] = clampq(round_int(subAmax[s] / (31.f * d)), subAmax[s] > 0 ? 1 : 0, 127);
    for (int w = 0; w < 256; w++) {
        int s = w / 16;
        float a = d * sc[s];
        int q = a > 0 ? clampq(round_int(x[w] / a) + 32, 0, 63) : 32;
        int lo = q & 0xF, hi = (q >> 4) & 3;
        int nn = (w / 128) * 128;
        int r = w - nn;
        int slot = r / 32, l = r % 32;
        if (slot == 0) y[nn / 2 + l] |= (uint8_t)lo;
        else if (slot == 1) y[nn / 2 + l + 32] |= (uint8_t)lo;
        else if (slot == 2) y[nn / 2 + l] |= (uint8_t)(lo << 4);
        else y[nn / 2 + l + 32] |= (uint8_t)(lo << 4);
        y[128 + nn / 4 + l] |= (uint8_t)(hi << (2 * slot));
    }
    for (int s = 0; s < 16; s++) y[192 + s] = (uint8_t)(int8_t)sc[s];
}

__device__ void tri_block(const float* x, uint8_t* y) {  // BlockQuantizer.cs:456-521
    float sorted[64];
    for (int i = 0; i < 18; i++) y[i] = 0;
    double energy = 0;
    float amax = 0.f;
    for (int i = 0; i < 64; i++) {
        float a = fabsf(x[i]);
        sorted[i] = a;
        energy += a * (double)a;
        if (a > amax) amax = a;
    }
    if (amax == 0.f) return;
    for (int i = 1; i < 64; i++) {  // ascending insertion sort
        float v = sorted[i];
        int j = i - 1;
        while (j >= 0 && sorted[j] > v) { sorted[j + 1] = sorted[j]; j--; }
        sorted[j + 1] = v;
    }
    double bestErr = 1.7976931348623157e308;
    float bestT = 0.f, bestAlpha = amax;
    for (int j = 0; j <= 60; j += 4) {
        float t = sorted[j];
        double sum = 0;
        int kept = 0;
        for (int i = 0; i < 64; i++)
            if (fabsf(x[i]) > t) { sum += fabsf(x[i]); kept++; }
        if (kept == 0) continue;
        float alpha = (float)(sum / kept);
        double err = energy - 2.0 * alpha * sum + (double)alpha * alpha * kept;
        if (err < bestErr) { bestErr = err; bestT = t; bestAlpha = alpha; }
    }
    {
        double sumAll = 0;
        for (int i = 0; i < 64; i++) sumAll += fabsf(x[i]);
        float tLegacy = (float)(sumAll / 64) * 0.5f;
        double sum = 0;
        int kept = 0;
        for (int i = 0; i < 64; i++)
            if (fabsf(x[i]) >= tLegacy) { sum += fabsf(x[i]); kept++; }
        if (kept > 0) {
            float alpha = (float)(sum / kept);
            double err = energy - 2.0 * alpha * sum + (double)alpha * alpha * kept;
            if (err < bestErr) { bestErr = err; bestT = tLegacy - 1e-9f; bestAlpha = alpha; }
        }
    }
    put16(y, f32_to_f16_ref(bestAlpha));
    for (int i = 0; i < 64; i++) {
        float a = fabsf(x[i]);
        int code = a > bestT ? (x[i] > 0 ? 1 : 2) : 0;
        y[2 + i / 4] |= (uint8_t)(code << (2 * (i & 3)));
    }
}

__device__ void tri_legacy_block(const float* x, uint8_t* y) {  // BlockQuantizer.cs:525-550
    for (int i = 0; i < 18; i++) y[i] = 0;
    double sum = 0;
    for (int i = 0; i < 64; i++) sum += fabsf(x[i]);
    float scale = (float)(sum / 64);
    if (scale == 0.f) return;
    put16(y, f32_to_f16_ref(scale));
    float iscale = 1.f / scale;
    for (int i = 0; i < 64; i++) {
        int v = round_int(x[i] * iscale);
        int code = v > 0 ? 1 : v < 0 ? 2 : 0;
        y[2 + i / 4] |= (uint8_t)(code << (2 * (i & 3)));
    }
}

// One thread per block.  Q4_K blocks start from zeroed codes; the CPU
// quantiser instead carries its code buffer over from the previous block, which
// differs only when a sub-block scale rounds to zero (a sub-block range below
// 1/126 of the block's largest range).  Gaussian weights never do that;
// tests/test_gpu_synth.py compares the bytes with the CPU quantiser.
__global__ void quantize_kernel(int fmt, const float* __restrict__ src, uint8_t* __restrict__ dst,
                                long long nb, int bs, int bb) {
    for (long long b = blockIdx.x * (long long)blockDim.x + threadIdx.x; b < nb;
         b += (long long)gridDim.x * blockDim.x) {
        const float* x = src + b * bs;
        uint8_t* y = dst + b * bb;
        switch (fmt) {
            case Q4_0: q4_0_block(x, y); break;
            case Q8_0: q8_0_block(x, y); break;
            case Q4_K: { uint8_t L[256]; for (int i = 0; i < 256; i++) L[i] = 0; q4_k_block(x, y, L); } break;
            case Q6_K: q6_k_block(x, y); break;
            case TRI: tri_block(x, y); break;
            case 108: tri_legacy_block(x, y); break;
            default: break;
        }
    }
}

}  // namespace qrm

extern "C" int qrm_synth_quantize_impl(int fmt, const float* src, long long n, void* dst, cudaStream_t s) {
    int f = fmt == 108 ? qrm::TRI : fmt;
    int bs, bb;
    if (!qrm::block_spec(f, &bs, &bb) || f == qrm::F32 || f == qrm::F16 || f == qrm::BF16) return QRM_E_FORMAT;
    if (n <= 0 || n % bs != 0) return QRM_E_INVALID;
    long long nb = n / bs;
    int threads = 128;
    long long blocks = (nb + threads - 1) / threads;
    if (blocks > 65535 * 16) blocks = 65535 * 16;
    qrm::quantize_kernel<<<(unsigned)blocks, threads, 0, s>>>(fmt, src, (uint8_t*)dst, nb, bs, bb);
    return cudaGetLastError() == cudaSuccess ? QRM_OK : QRM_E_CUDA;
}

extern "C" int qrm_synth_gaussian_impl(float* dst, long long n, uint64_t seed, float sigma, cudaStream_t s) {
    if (n <= 0) return QRM_E_INVALID;
    long long blocks = (n + 255) / 256;
    if (blocks > 148 * 64) blocks = 148 * 64;
    qrm::gaussian_kernel<<<(unsigned)blocks, 256, 0, s>>>(dst, n, seed, sigma);
    return cudaGetLastError() == cudaSuccess ? QRM_OK : QRM_E_CUDA;
}
