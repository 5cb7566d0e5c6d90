// gemv_imma.cuh -- building blocks of the integer tensor-core expert kernel
// (gemv_stream.cuh).
//
// The expert matrices stay in their integer codes: a Q4_K / Q4_0 nibble or a
// Q8_0 byte is fed to mma.sync m16n8k32 as an 8-bit operand after one mask
// (no conversion to float).  Activations are quantised per 32-weight group to
// 16-bit fixed point x = s * (256*hi + lo) with hi int8, lo uint8 (|error| <=
// s/2 = amax/65534, about 5 significant digits), so each group product is two
// exact integer MMAs.  The per-group scales of the weights (Q4_K: d*sc and
// dmin*m of 32-weight sub-blocks; Q4_0/Q8_0: d) are applied in f32 afterwards.
//
// Decode layout (one token, "diagonal" B): four groups of 32 weights are four
// MMAs whose B operand is non-zero only in the column pair of its group, so
// the 16x8 accumulator holds the group sums (hi and lo parts) of 16 rows at
// once.  Several tokens repeat the MMAs with their own activations.
//
// This file: the MMA wrappers, the activation tables and their quantiser,
// bounded waits and shared-memory loads.
#pragma once
#include <algorithm>
#include <cstdlib>

#include "common.cuh"
#include "gemv.cuh"
#include "gemv_tma.cuh"

namespace qrm {

__device__ __forceinline__ void mma_u8s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_u8u8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_s8s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_s8u8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// ------------------------------------------------------------ activations
// Per token row: hi[K] int8 | 64 bytes | lo[K] int8 | 64 bytes | ss[K/32]
// float2 (scale s, sum of the group's original f32 values for the Q4_K / Q4_0
// min terms).  The 64-byte gaps put the hi and lo bytes that a half warp reads
// together on distinct banks.
constexpr int kXtabLo = 64;
__host__ __device__ inline int xtab_lo(int K) { return K + kXtabLo; }
__host__ __device__ inline int xtab_ss(int K) { return 2 * K + 2 * kXtabLo; }
__host__ __device__ inline int xtab_bytes(int K) { return xtab_ss(K) + 8 * (K / 32); }
inline int xtab_stride(int K) { return (xtab_bytes(K) + 15) / 16 * 16; }

// Quantises four consecutive 32-element groups of one activation row, one
// warp: lane l holds elements 4(l%8)..+3 of group 4c + l/8 (v), and writes the
// table row at `row` (global or shared memory): q = rint(x * 32639 / amax),
// s = amax / 32639 per group, hi = floor((q + 128) / 256) in [-127, 127], lo = q - 256 hi
// in [-128, 127], ss = (s, sum of the group's values).
__device__ __forceinline__ void xquant_quad(float4 v, int lane, int c, int K, uint8_t* row) {
    float amax = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
    float sum = (v.x + v.y) + (v.z + v.w);
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) {
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        sum += __shfl_xor_sync(0xffffffffu, sum, o);
    }
    const float s = amax > 0.f ? amax * (1.f / 32639.f) : 0.f;
    const float inv = amax > 0.f ? 32639.f / amax : 0.f;   // one division per group
    const float vv[4] = {v.x, v.y, v.z, v.w};
    uint32_t hw = 0, lw = 0;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        int q = __float2int_rn(vv[i] * inv);
        q = max(-32639, min(32639, q));
        const int hi = (q + 128) >> 8;   // arithmetic shift: floor
        hw |= (uint32_t)(uint8_t)(int8_t)hi << (8 * i);
        lw |= (uint32_t)(uint8_t)(int8_t)(q - 256 * hi) << (8 * i);
    }
    const int g = 4 * c + (lane >> 3), off = 32 * g + 4 * (lane & 7);
    *reinterpret_cast<uint32_t*>(row + off) = hw;
    *reinterpret_cast<uint32_t*>(row + xtab_lo(K) + off) = lw;
    if ((lane & 7) == 0) reinterpret_cast<float2*>(row + xtab_ss(K))[g] = make_float2(s, sum);
}

// The same for one 32-element group gi, lane l holding element l.
__device__ __forceinline__ void xquant_group(float v, int lane, int gi, int K, uint8_t* row) {
    float amax = fabsf(v), sum = v;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        sum += __shfl_xor_sync(0xffffffffu, sum, o);
    }
    const float s = amax > 0.f ? amax * (1.f / 32639.f) : 0.f;
    const float inv = amax > 0.f ? 32639.f / amax : 0.f;
    int q = __float2int_rn(v * inv);
    q = max(-32639, min(32639, q));
    const int hi = (q + 128) >> 8;
    row[gi * 32 + lane] = (uint8_t)(int8_t)hi;
    row[xtab_lo(K) + gi * 32 + lane] = (uint8_t)(int8_t)(q - 256 * hi);
    if (lane == 0) reinterpret_cast<float2*>(row + xtab_ss(K))[gi] = make_float2(s, sum);
}

// Quantises activation rows into tables (global memory), one warp per four
// groups (K % 128 == 0).  Rows below `split` come from src, the others from
// src_b (row r - split): the routed and the shared rows of one stage in one
// launch.
static __global__ void xquant_kernel(const float* __restrict__ src, const float* __restrict__ src_b, int split, int K,
                                     int rows, uint8_t* __restrict__ tab, int stride) {
    const int lane = threadIdx.x & 31;
    const int quads = K / 128;
    const long long total = (long long)rows * quads;
    for (long long w = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5; w < total;
         w += ((long long)gridDim.x * blockDim.x) >> 5) {
        const int r = (int)(w / quads), c = (int)(w - (long long)r * quads);
        const float* row = r < split ? src + (size_t)r * K : src_b + (size_t)(r - split) * K;
        const float4 v = reinterpret_cast<const float4*>(row)[32 * c + lane];
        xquant_quad(v, lane, c, K, tab + (size_t)r * stride);
    }
}

// ------------------------------------------------------------ bounded waits
// Every wait gives up after wait_limit_ns() or as soon as another warp of the
// CTA has given up (abort flag), so no warp can wait forever on one that left.
// try_wait carries a suspend-time hint so a waiting warp sleeps instead of
// taking issue slots from the warps that compute.
constexpr uint32_t kSuspendHintNs = 20000;
__device__ __forceinline__ bool mbar_try_wait_hint(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendHintNs)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_abort(uint64_t* bar, uint32_t parity, const volatile int* abort_flag) {
    if (mbar_try_wait_hint(bar, parity)) return true;
    const uint64_t t0 = global_ns(), lim = wait_limit_ns();
    for (;;) {
        for (int i = 0; i < 4; i++)
            if (mbar_try_wait_hint(bar, parity)) return true;
        if (*abort_flag) return false;
        if (global_ns() - t0 > lim) return false;
    }
}
// whole warp; false (for every lane) when any lane gave up
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int32_t* err) {
    const bool ok = __all_sync(0xffffffffu, mbar_wait_abort(bar, parity, abort_flag));
    if (!ok && (threadIdx.x & 31) == 0) {
        *abort_flag = 1;
        atomicOr(err, (int)ERR_TIMEOUT);
    }
    return ok;
}
// lane 0 spins (with a short back-off, so the waiting warp leaves the issue
// slots to the others) until *f == v; whole warp returns the outcome
__device__ __forceinline__ bool warp_spin_eq(const volatile int* f, int v, volatile int* abort_flag, int32_t* err) {
    int ok = 1;
    if ((threadIdx.x & 31) == 0) {
        const uint64_t t0 = global_ns(), lim = wait_limit_ns();
        while (*f != v) {
            __nanosleep(32);
            if (*abort_flag || global_ns() - t0 > lim) { ok = 0; break; }
        }
        if (!ok) {
            *abort_flag = 1;
            atomicOr(err, (int)ERR_TIMEOUT);
        }
        __threadfence_block();
    }
    ok = __shfl_sync(0xffffffffu, ok, 0);
    __syncwarp();
    return ok != 0;
}

// ------------------------------------------------------------ shared loads
// 32-bit shared addresses keep the per-super-block address arithmetic to
// plain adds.  volatile: the stage bytes are written by the bulk copies,
// which the compiler does not see, so no load may move above the waits.
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t a) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}
__device__ __forceinline__ uint4 lds128(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
__device__ __forceinline__ uint32_t lds16(uint32_t a) {
    uint16_t v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
    return v;
}
// activation-table loads: shared (resident or staged tables) or global
template <bool SM> struct TabLd;
template <> struct TabLd<true> {
    using Ptr = const uint8_t*;
    __device__ static uint32_t ld32(Ptr b, int o) { return lds32(smem_u32(b) + o); }
    __device__ static uint2 ld64(Ptr b, int o) { return lds64(smem_u32(b) + o); }
};
template <> struct TabLd<false> {
    using Ptr = const uint8_t*;
    __device__ static uint32_t ld32(Ptr b, int o) { return __ldg(reinterpret_cast<const uint32_t*>(b + o)); }
    __device__ static uint2 ld64(Ptr b, int o) { return __ldg(reinterpret_cast<const uint2*>(b + o)); }
};

}  // namespace qrm
