// gemv_imma.cuh -- decode-size expert products on the integer tensor cores.
//
// The expert matrices stay in their integer codes: a Q4_K / Q4_0 nibble or a
// Q8_0 byte is fed to mma.sync m16n8k32 as an 8-bit operand after one mask
// (no conversion to float).  Activations are quantised per 32-weight group to
// 16-bit fixed point x = s * (256*hi + lo) with hi int8, lo uint8 (|error| <=
// s/2 = amax/65534, about 5 significant digits), so each group product is two
// exact integer MMAs.  The per-group scales of the weights (Q4_K: d*sc and
// dmin*m of 32-weight sub-blocks; Q4_0/Q8_0: d) are applied in f32 afterwards.
//
// Decode layout (one token, "diagonal" B): a super-block of 8 groups (256
// weights) is 8 MMAs whose B operand is non-zero only in column j = group j,
// so the 16x8 accumulator holds the 8 group sums of 16 rows at once and the
// f32 scale epilogue runs once per super-block.  Several tokens repeat the
// MMAs with their own activations and accumulators.
//
// Data movement is the bulk-copy pipeline of gemv_tma.cuh: a producer warp
// copies the 16 rows of an item (8 gate + 8 up rows, or 16 down rows) into a
// shared-memory stage with a 16-byte row padding (bank-conflict-free fragment
// loads); consumer warps split the K dimension, reduce across warps in a fixed
// order, and apply SwiGLU.  All waits are bounded.
#pragma once
#include <algorithm>
#include <cstdlib>

#include "common.cuh"
#include "gemv.cuh"
#include "gemv_tma.cuh"

namespace qrm {

__device__ __forceinline__ void mma_u8s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_u8u8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_s8s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_s8u8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
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
// groups (K % 128 == 0).
__global__ void xquant_kernel(const float* __restrict__ src, int K, int rows, uint8_t* __restrict__ tab,
                              int stride) {
    const int lane = threadIdx.x & 31;
    const int quads = K / 128;
    const long long total = (long long)rows * quads;
    for (long long w = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5; w < total;
         w += ((long long)gridDim.x * blockDim.x) >> 5) {
        const int r = (int)(w / quads), c = (int)(w - (long long)r * quads);
        const float4 v = reinterpret_cast<const float4*>(src + (size_t)r * K)[32 * c + lane];
        xquant_quad(v, lane, c, K, tab + (size_t)r * stride);
    }
}

// ------------------------------------------------------------ formats

template <int FMT> struct ImmaFmt;

// Q4_K: 144-byte blocks (d, dmin, scales[12], qs[128]); group g of a block =
// nibble (g & 1) of qs bytes [32*(g>>1), +32).  Lane t takes bytes [8t, 8t+8)
// of the group: K slots 4t..4t+3 <- bytes 8t..8t+3, 16+4t.. <- 8t+4..8t+7.
template <> struct ImmaFmt<Q4_K> {
    static constexpr int kBS = 256;          // weights per block
    static constexpr int kFields = 1;
    __host__ __device__ static int len(int) { return 144; }
    __host__ __device__ static long long base_mul(int) { return 0; }
};
// Q8_0 (split layout): qs[nb][32] | d[nb]; group = block of 32 int8 codes.
template <> struct ImmaFmt<Q8_0> {
    static constexpr int kBS = 32;
    static constexpr int kFields = 2;
    __host__ __device__ static int len(int f) { return f == 0 ? 32 : 2; }
    __host__ __device__ static long long base_mul(int f) { return f == 0 ? 0 : 32; }
};
// Q4_0 (split layout): qs[nb][16] | d[nb] | pad; group = block of 32 nibbles,
// low nibble of byte i = weight i, high nibble = weight 16+i, y = d*(q-8).
template <> struct ImmaFmt<Q4_0> {
    static constexpr int kBS = 32;
    static constexpr int kFields = 2;
    __host__ __device__ static int len(int f) { return f == 0 ? 16 : 2; }
    __host__ __device__ static long long base_mul(int f) { return f == 0 ? 0 : 16; }
};

// ------------------------------------------------------------ stage plan

constexpr int kImmaRows = 16;                 // MMA rows per row tile
constexpr int kImmaMaxTok = 2;                // most tokens per pass
constexpr int kImmaMaxWarps = 16;             // consumer warps (one token per pass)
constexpr int kImmaMaxWarps2 = 15;            // consumer warps (two tokens per pass)
constexpr int kImmaMaxSplit = 4;              // K parts of a shared-expert item
// per-stage header: item, slot, e, off, n_tok, (unused x2), segment, part,
// tile, table rows of the first two tokens
constexpr int kImmaHdrInts = 12;
constexpr int kImmaCtlOff = 8 * (2 * kTmaMaxStages + 1);   // after full[], empty[], the table barrier
constexpr int kImmaHdrOff = 256;
constexpr int kImmaDataOff = (kImmaHdrOff + kTmaMaxStages * kImmaHdrInts * 4 + 127) / 128 * 128;
static_assert(kImmaCtlOff + 48 + 48 <= kImmaHdrOff, "imma control area: abort flag, arrivals, tickets, next item");

// bytes of field f of a format per super-block of 256 columns
__host__ __device__ inline int imma_sb_bytes(int fmt, int f) {
    switch (fmt) {
        case Q4_K: return f == 0 ? 144 : 0;
        case Q8_0: return f == 0 ? 256 : 16;
        case Q4_0: return f == 0 ? 128 : 16;
        default: return 0;
    }
}

// Whole-row items are copied as one bulk copy per run of consecutive rows
// into unpadded rows (few large copies keep HBM busier than many padded row
// copies, at the price of bank conflicts); QRM_IMMA_CONTIG=0 pads every row.
__host__ inline bool imma_contig() {
    static int v = -1;
    if (v < 0) {
        const char* e = getenv("QRM_IMMA_CONTIG");
        v = (e && e[0] == '0') ? 0 : 1;
    }
    return v == 1;
}

// Stage geometry of one segment of a launch (0: routed experts, 1: the shared
// expert).  An item of the segment is cut into nsplit parts along K.
struct ImmaSeg {
    int nsplit;          // K parts per item (1: whole rows)
    int pitch[2];        // bytes between rows of field f in a stage
    int field_off[2];    // offset of field f's row 0 in a stage
    int row_bytes[2];    // bytes of a whole matrix row of field f
    int part_bytes[2];   // bytes of field f copied per row for one part
    int nsbp;            // super-blocks per part
    int contig;          // whole rows, unpadded: one bulk copy per run of consecutive rows
};

constexpr int kImmaRedSlots = 4;              // reduction slots (items in reduction at once)

struct ImmaConfig {
    int stages;
    int stage_bytes;     // weights (+ per-item tables)
    ImmaSeg seg[2];
    int xtab_bytes;      // per token table (16-byte multiple)
    int xtab_off;        // per-item tables inside a stage (resident: unused)
    int res_rows;        // > 0: all table rows resident in shared memory
    int red_bytes;       // one reduction slot: partial sums [warps][NTK][16] floats
};

// Returns the weight bytes of a stage, -1 when a part of a field is not a
// multiple of 16 bytes (bulk copies).  Row pitch = 32 or 96 mod 128: the
// 8-byte fragment loads of a half warp (4 rows x 32 bytes) hit distinct banks.
__host__ inline int imma_seg_geom(int fmt, int cols, int rows, int nsplit, ImmaSeg* g, bool contig) {
    const int nsb = cols / 256;
    if (nsplit < 1 || nsb % nsplit) return -1;
    int off = 0;
    g->nsplit = nsplit;
    g->nsbp = nsb / nsplit;
    g->contig = contig && nsplit == 1;
    for (int f = 0; f < 2; f++) {
        const int b = imma_sb_bytes(fmt, f);
        g->row_bytes[f] = nsb * b;
        g->part_bytes[f] = nsb / nsplit * b;
        if (g->part_bytes[f] % 16) return -1;
        const int m = g->part_bytes[f] % 128;
        g->pitch[f] = !b ? 0 : g->contig ? g->part_bytes[f]
                                         : g->part_bytes[f] + (m <= 32 ? 32 - m : (m <= 96 ? 96 - m : 160 - m));
        g->field_off[f] = off;
        off += rows * g->pitch[f];
    }
    return off;
}

// fmt[0] / fmt[1]: formats of the routed and the shared segment (-1: none in
// this launch).  Routed items take whole rows; shared items are split along K
// until their stage is no larger than the routed one (alone: until two stages
// fit).  tab_rows = table rows the launch reads.  Tables are kept resident
// when that costs no pipeline depth (at least min(4, per-item stages) stages);
// split items need them resident.
__host__ inline bool imma_plan(const int (&fmt)[2], int cols, int rows_per_item, int ntok, int cw, int tab_rows,
                               int smem_budget, ImmaConfig* c) {
    if (cols % 256) return false;
    const int nsb = cols / 256;
    const int red = cw * ntok * 16 * 4;
    const int avail = smem_budget - kImmaDataOff;
    int wbytes = 0;
    c->seg[0] = ImmaSeg{};
    c->seg[1] = ImmaSeg{};
    c->seg[0].nsplit = c->seg[1].nsplit = 1;
    if (fmt[0] >= 0) {
        wbytes = imma_seg_geom(fmt[0], cols, rows_per_item, 1, &c->seg[0], imma_contig());
        if (wbytes < 0) return false;
    }
    if (fmt[1] >= 0) {
        const int target = fmt[0] >= 0 ? wbytes : (avail - red) / 2;
        int b = -1;
        for (int sp = 1; sp <= kImmaMaxSplit && b < 0; sp++) {
            b = imma_seg_geom(fmt[1], cols, rows_per_item, sp, &c->seg[1], imma_contig());
            if (b > target) b = -1;
        }
        if (b < 0) return false;
        wbytes = std::max(wbytes, b);
    }
    const bool split = c->seg[1].nsplit > 1;
    c->xtab_bytes = xtab_stride(cols);
    c->red_bytes = red;
    const int avail2 = avail - kImmaRedSlots * red;
    const long long res = (long long)tab_rows * c->xtab_bytes;
    const int stA = wbytes;
    const int sA = res < avail2 ? (int)std::min<long long>(kTmaMaxStages, (avail2 - res) / stA) : 0;
    const int stB = wbytes + ntok * c->xtab_bytes;
    const int sB = std::min(kTmaMaxStages, avail2 / stB);
    if (tab_rows > 0 && sA >= 2 && (split || sA >= std::min(sB, 4))) {
        c->res_rows = tab_rows;
        c->xtab_off = 0;
        c->stage_bytes = stA;
        c->stages = sA;
    } else if (!split && sB >= 2) {
        c->res_rows = 0;
        c->xtab_off = wbytes;
        c->stage_bytes = stB;
        c->stages = sB;
    } else {
        return false;
    }
    return true;
}
// shared memory: control | resident tables | reduction slots | stages
inline size_t imma_smem_bytes(const ImmaConfig& c) {
    return (size_t)kImmaDataOff + (size_t)c.res_rows * c.xtab_bytes + (size_t)kImmaRedSlots * c.red_bytes +
           (size_t)c.stages * c.stage_bytes;
}

// ------------------------------------------------------------ bounded waits
// Every wait gives up after kWaitLimitNs or as soon as another warp of the CTA
// has given up (abort flag), so no warp can wait forever on one that left.
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
    const uint64_t t0 = global_ns();
    for (;;) {
        for (int i = 0; i < 4; i++)
            if (mbar_try_wait_hint(bar, parity)) return true;
        if (*abort_flag) return false;
        if (global_ns() - t0 > kWaitLimitNs) return false;
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
// lane 0 spins until *f == v; whole warp returns the outcome
__device__ __forceinline__ bool warp_spin_eq(const volatile int* f, int v, volatile int* abort_flag, int32_t* err) {
    int ok = 1;
    if ((threadIdx.x & 31) == 0) {
        const uint64_t t0 = global_ns();
        while (*f != v) {
            if (*abort_flag || global_ns() - t0 > kWaitLimitNs) { ok = 0; break; }
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
    using Ptr = uint32_t;
    __device__ static uint32_t ld32(Ptr b, int o) { return lds32(b + o); }
    __device__ static uint2 ld64(Ptr b, int o) { return lds64(b + o); }
};
template <> struct TabLd<false> {
    using Ptr = const uint8_t*;
    __device__ static uint32_t ld32(Ptr b, int o) { return __ldg(reinterpret_cast<const uint32_t*>(b + o)); }
    __device__ static uint2 ld64(Ptr b, int o) { return __ldg(reinterpret_cast<const uint2*>(b + o)); }
};

// ------------------------------------------------------------ one pass
// Accumulates this warp's K slice [sb0, sb1) (super-blocks of the stage) of
// rows gid / gid+8 of its row tile for nt <= NTK tokens whose tables start at
// tq[q]; stage super-block sb is table super-block sb + sb_tab.  y[q][0] = row gid,
// y[q][1] = row gid+8 (this lane's two groups t and t+4 only).  r0 / d0: shared
// addresses of row gid of field 0 / field 1 (row gid+8 is 8 pitches on).
template <int FMT, int NTK, bool SM>
__device__ __forceinline__ void imma_pass(uint32_t r0, uint32_t pitch0, uint32_t d0, uint32_t pitch1,
                                          const typename TabLd<SM>::Ptr (&tq)[NTK], int nt, int K, int sb0,
                                          int sb1, int sb_tab, int lane, const uint32_t (&bm)[4],
                                          float (&y)[NTK][2]) {
    using L = TabLd<SM>;
    const int gid = lane >> 2, t = lane & 3, j = gid >> 1, hl = gid & 1;
    // Q4_K: odd groups (high nibbles) keep the nibble in place (code * 16)
    const float kq = (FMT == Q4_K && (t & 1)) ? 4.f : 64.f;
    const uint32_t sel = 0x7044u | ((uint32_t)t << 8);   // byte t -> bits 16..23 of 2.0f
    const uint32_t r1 = r0 + 8 * pitch0, d1 = d0 + 8 * pitch1;
    const int bofs = hl * xtab_lo(K) + 32 * j + (FMT == Q4_0 ? 4 : 8) * t + 256 * sb_tab;   // this lane's B bytes
    const int sofs = xtab_ss(K) + 8 * t + 64 * sb_tab;                                        // its ss entry
#pragma unroll
    for (int q = 0; q < NTK; q++) y[q][0] = y[q][1] = 0.f;
    for (int sb = sb0; sb < sb1; sb++) {
        // B bytes of groups j and j+4 (this lane's half: hi or lo); zero for
        // tokens past nt so the MMAs can run unconditionally
        uint32_t bx[NTK][2][2];
#pragma unroll
        for (int q = 0; q < NTK; q++) {
            const int o = bofs + 256 * sb;
            if (q == 0 || q < nt) {
                if (FMT == Q4_0) {
                    bx[q][0][0] = L::ld32(tq[q], o);
                    bx[q][0][1] = L::ld32(tq[q], o + 16);
                    bx[q][1][0] = L::ld32(tq[q], o + 128);
                    bx[q][1][1] = L::ld32(tq[q], o + 144);
                } else {
                    const uint2 a = L::ld64(tq[q], o);
                    const uint2 b = L::ld64(tq[q], o + 128);
                    bx[q][0][0] = a.x; bx[q][0][1] = a.y; bx[q][1][0] = b.x; bx[q][1][1] = b.y;
                }
            } else {
                bx[q][0][0] = bx[q][0][1] = bx[q][1][0] = bx[q][1][1] = 0u;
            }
        }
        int X[NTK][4], Y[NTK][4];
#pragma unroll
        for (int q = 0; q < NTK; q++)
#pragma unroll
            for (int i = 0; i < 4; i++) X[q][i] = Y[q][i] = 0;
#pragma unroll
        for (int pr = 0; pr < 4; pr++) {
            uint32_t A0[4], A1[4];   // groups 2pr, 2pr+1
            if (FMT == Q4_K) {
                const uint32_t o = 144 * sb + 16 + 32 * pr + 8 * t;
                const uint2 w0 = lds64(r0 + o);
                const uint2 w1 = lds64(r1 + o);
                A0[0] = w0.x & 0x0F0F0F0Fu; A0[1] = w1.x & 0x0F0F0F0Fu; A0[2] = w0.y & 0x0F0F0F0Fu; A0[3] = w1.y & 0x0F0F0F0Fu;
                A1[0] = w0.x & 0xF0F0F0F0u; A1[1] = w1.x & 0xF0F0F0F0u; A1[2] = w0.y & 0xF0F0F0F0u; A1[3] = w1.y & 0xF0F0F0F0u;
            } else if (FMT == Q8_0) {
                const uint32_t o = 256 * sb + 64 * pr + 8 * t;
                const uint2 a0 = lds64(r0 + o), a1 = lds64(r1 + o);
                const uint2 b0 = lds64(r0 + o + 32), b1 = lds64(r1 + o + 32);
                A0[0] = a0.x; A0[1] = a1.x; A0[2] = a0.y; A0[3] = a1.y;
                A1[0] = b0.x; A1[1] = b1.x; A1[2] = b0.y; A1[3] = b1.y;
            } else {  // Q4_0
                const uint32_t o = 128 * sb + 32 * pr + 4 * t;
                const uint32_t a0 = lds32(r0 + o), a1 = lds32(r1 + o);
                const uint32_t b0 = lds32(r0 + o + 16), b1 = lds32(r1 + o + 16);
                A0[0] = a0 & 0x0F0F0F0Fu; A0[1] = a1 & 0x0F0F0F0Fu;
                A0[2] = (a0 >> 4) & 0x0F0F0F0Fu; A0[3] = (a1 >> 4) & 0x0F0F0F0Fu;
                A1[0] = b0 & 0x0F0F0F0Fu; A1[1] = b1 & 0x0F0F0F0Fu;
                A1[2] = (b0 >> 4) & 0x0F0F0F0Fu; A1[3] = (b1 >> 4) & 0x0F0F0F0Fu;
            }
#pragma unroll
            for (int half = 0; half < 2; half++) {
                const int g = 2 * pr + half;
                const uint32_t(&A)[4] = half ? A1 : A0;
#pragma unroll
                for (int q = 0; q < NTK; q++) {
                    const uint32_t b0 = bx[q][g >> 2][0] & bm[g & 3], b1 = bx[q][g >> 2][1] & bm[g & 3];
                    if (FMT == Q8_0) {
                        if (g < 4) mma_s8s8(X[q], A, b0, b1); else mma_s8s8(Y[q], A, b0, b1);
                    } else {
                        if (g < 4) mma_u8s8(X[q], A, b0, b1); else mma_u8s8(Y[q], A, b0, b1);
                    }
                }
            }
        }
        // scales of groups t (X) and t+4 (Y) for rows gid, gid+8:
        // y += a * (c * s) - mm * sum
        float ar[2][2], mr[2][2];
        if (FMT == Q4_K) {
#pragma unroll
            for (int rw = 0; rw < 2; rw++) {
                const uint4 hd = lds128((rw ? r1 : r0) + 144 * sb);
                const float d = h2f((uint16_t)(hd.x & 0xFFFF)), dmin = h2f((uint16_t)(hd.x >> 16));
                // GetScaleMinK4 (BlockDequantizer.cs:155-166), four sub-blocks per word:
                // sc[0..3] = q[0..3] & 63, m[0..3] = q[4..7] & 63,
                // sc[4..7] = (q[8..11] & 15) | (q[0..3] >> 6) << 4, m[4..7] = (q[8..11] >> 4) | (q[4..7] >> 6) << 4
                const uint32_t SC0 = hd.y & 0x3F3F3F3Fu, MN0 = hd.z & 0x3F3F3F3Fu;
                const uint32_t SC1 = (hd.w & 0x0F0F0F0Fu) | ((hd.y >> 2) & 0x30303030u);
                const uint32_t MN1 = ((hd.w >> 4) & 0x0F0F0F0Fu) | ((hd.z >> 2) & 0x30303030u);
                // byte b at bits 16..23 of 2.0f reads 2 + b/64: d*b = F*64d - 128d (the
                // high-nibble groups take another 1/16)
                const float da = kq * d, db = -2.f * kq * d, ma = 64.f * dmin, mb = -128.f * dmin;
                ar[rw][0] = fmaf(__uint_as_float(prmt(SC0, 0x40000000u, sel)), da, db);
                ar[rw][1] = fmaf(__uint_as_float(prmt(SC1, 0x40000000u, sel)), da, db);
                mr[rw][0] = fmaf(__uint_as_float(prmt(MN0, 0x40000000u, sel)), ma, mb);
                mr[rw][1] = fmaf(__uint_as_float(prmt(MN1, 0x40000000u, sel)), ma, mb);
            }
        } else {
#pragma unroll
            for (int i = 0; i < 2; i++) {
                const uint32_t o = 16 * sb + 2 * t + 8 * i;   // block 8sb + t + 4i
                const float dA = h2f((uint16_t)lds16(d0 + o));
                const float dB = h2f((uint16_t)lds16(d1 + o));
                ar[0][i] = dA; ar[1][i] = dB;
                mr[0][i] = FMT == Q4_0 ? 8.f * dA : 0.f;
                mr[1][i] = FMT == Q4_0 ? 8.f * dB : 0.f;
            }
        }
#pragma unroll
        for (int q = 0; q < NTK; q++) {
            if (q == 0 || q < nt) {
                const uint2 u0 = L::ld64(tq[q], sofs + 64 * sb), u1 = L::ld64(tq[q], sofs + 64 * sb + 32);
                const float2 s0 = make_float2(__uint_as_float(u0.x), __uint_as_float(u0.y));
                const float2 s1 = make_float2(__uint_as_float(u1.x), __uint_as_float(u1.y));
                const float c00 = (float)(X[q][0] * 256 + X[q][1]), c10 = (float)(X[q][2] * 256 + X[q][3]);
                const float c01 = (float)(Y[q][0] * 256 + Y[q][1]), c11 = (float)(Y[q][2] * 256 + Y[q][3]);
                float a = y[q][0], b = y[q][1];
                a = fmaf(ar[0][0], c00 * s0.x, a);
                a = fmaf(ar[0][1], c01 * s1.x, a);
                b = fmaf(ar[1][0], c10 * s0.x, b);
                b = fmaf(ar[1][1], c11 * s1.x, b);
                if (FMT != Q8_0) {
                    a = fmaf(-mr[0][0], s0.y, a);
                    a = fmaf(-mr[0][1], s1.y, a);
                    b = fmaf(-mr[1][0], s0.y, b);
                    b = fmaf(-mr[1][1], s1.y, b);
                }
                y[q][0] = a;
                y[q][1] = b;
            }
        }
    }
}

// ------------------------------------------------------------ kernel
// Item = (segment, slot, row tile group, K part).  A row tile group is RTILES
// row tiles of 16 MMA rows: gate/up (M = 2): 8 rows of gate and the same 8
// rows of up (a thread holds gate row g and up row g); down (M = 1): 16
// consecutive rows.  CW consumer warps (blockDim/32 - 1): warp w takes row
// tile w % RTILES and K slice w / RTILES of the part.  The producer warp
// resolves each item (expert, token run), copies its weight rows (and, when the
// tables are not resident, the first NTK tables) into the stage and writes the
// item header, S stages ahead of the consumers.  Routed items use format FA,
// the shared expert's items FB.

// Producer: this lane's share of the row copies of one item.
template <int FMT, int M, int RTILES>
__device__ __forceinline__ void imma_issue(const GemvParams& p, const ImmaSeg& g, const MatDev* md, int tile,
                                           int part, uint8_t* st, uint64_t* bar, int lane) {
    using F = ImmaFmt<FMT>;
    constexpr int RT = kImmaRows / M, ROWS = kImmaRows * RTILES;
    if (g.contig) {
        // runs: down, all ROWS rows of the matrix; gate/up, per row tile the RT
        // rows of gate and of up
        constexpr int RUNS = M == 2 ? 2 * RTILES : 1, RUN = M == 2 ? RT : ROWS;
        for (int c = lane; c < RUNS * F::kFields; c += 32) {
            const int f = c / RUNS, run = c - f * RUNS;
            const int m = M == 2 ? run & 1 : 0, rt = M == 2 ? run >> 1 : 0;
            const MatDev mat = md[M == 2 ? m : 2];
            const int row = M == 2 ? (tile * RTILES + rt) * RT : tile * ROWS;
            const int r = M == 2 ? rt * kImmaRows + m * RT : 0;   // first stage row of the run
            const uint8_t* src = mat.base + mat.nb * F::base_mul(f) + (size_t)row * g.row_bytes[f];
            bulk_g2s(st + g.field_off[f] + r * g.pitch[f], src, (uint32_t)(RUN * g.row_bytes[f]), bar);
        }
        return;
    }
    for (int c = lane; c < ROWS * F::kFields; c += 32) {
        const int f = c / ROWS, r = c - f * ROWS;
        const int rt = r / kImmaRows, rr = r % kImmaRows;
        const MatDev mat = md[M == 2 ? rr / RT : 2];
        const int row = (tile * RTILES + rt) * RT + (rr % RT);
        const uint8_t* src = mat.base + mat.nb * F::base_mul(f) + (size_t)row * g.row_bytes[f] + (size_t)part * g.part_bytes[f];
        bulk_g2s(st + g.field_off[f] + r * g.pitch[f], src, (uint32_t)g.part_bytes[f], bar);
    }
}

// Fused combine of one finished down item (one warp): counts the item against
// its row tile; the last of the tile's n_active + shared items writes
// out[t][tile columns] = x + w_0 y_0 + ... + w_{k-1} y_{k-1} + ys for every
// token, each term separately rounded in slot order as combine_kernel does.
template <int OUTS>
__device__ __forceinline__ void imma_combine_tile(const GemvParams& p, int tile, int n_active, int lane) {
    __threadfence();
    __syncwarp();
    int last = 0;
    if (lane == 0) last = atomicAdd(&p.tile_ctr[tile], 1) == n_active + (p.has_shared ? 1 : 0) - 1;
    last = __shfl_sync(0xffffffffu, last, 0);
    if (!last) return;
    __threadfence();
    const int d = p.rows;
    for (int o = lane; o < p.T * OUTS; o += 32) {
        const int t = o / OUTS, col = tile * OUTS + (o - t * OUTS);
        float acc = p.cmb_x ? __ldcg(p.cmb_x + (size_t)t * d + col) : 0.f;
        for (int j = 0; j < p.k; j++) {
            const float w = __ldcg(p.cmb_w + t * p.k + j);
            const int pos = __ldcg(p.cmb_inv + t * p.k + j);
            acc = __fadd_rn(acc, __fmul_rn(w, __ldcg(p.out_routed + (size_t)pos * d + col)));
        }
        if (p.has_shared) acc = __fadd_rn(acc, __ldcg(p.out_shared + (size_t)t * d + col));
        p.cmb_out[(size_t)t * d + col] = acc;
    }
    __syncwarp();
    if (lane == 0) p.tile_ctr[tile] = 0;
}

// Per-CTA reduction state: kImmaRedSlots slots of partial sums; reduction r
// of the CTA (items, and passes within an item, in order) uses slot r % slots
// once the slot's ticket shows the reductions before it are done.
struct ImmaRed {
    int* arr;     // [slots] warps arrived with their partials
    int* tick;    // [slots] reductions completed in the slot
    float* buf;   // [slots][red floats]
    int floats;   // floats per slot
};

// What a reduction needs once the stage and its header are gone.
struct ImmaRedJob;
template <int OUTS>
__device__ __forceinline__ void imma_qgroups(const GemvParams& p, const ImmaRedJob& j, int lane);

struct ImmaRedJob {
    int r;          // reduction number (slot r % kImmaRedSlots); -1: none
    int seg, part, tile, off, t0, nt;
    int shared, final_pass;
};

// Gate/up outputs of job j are written: count them against their 32-output
// groups (per token row); the writer of a group's last tile quantises the
// group into the down launch's table row (routed rows = output rows, shared
// rows after the T*k routed ones).
template <int OUTS>
__device__ __forceinline__ void imma_qgroups(const GemvParams& p, const ImmaRedJob& j, int lane) {
    const int f = p.rows, ng = f / 32;
    __threadfence();
    __syncwarp();
    for (int q = 0; q < j.nt; q++) {
        const int tk = j.t0 + q;
        const int trow = j.shared ? p.T * p.k + tk : j.off + tk;
        const float* hrow = j.shared ? p.out_shared + (size_t)tk * f : p.out_routed + (size_t)(j.off + tk) * f;
        uint8_t* qrow = p.qtab + (size_t)trow * p.qtab_stride;
        if (OUTS >= 32) {
            for (int g = j.tile * (OUTS / 32); g < (j.tile + 1) * (OUTS / 32); g++)
                xquant_group(__ldcg(hrow + 32 * g + lane), lane, g, f, qrow);
        } else {
            const int g = j.tile * OUTS / 32;
            int last = 0;
            if (lane == 0) last = atomicAdd(&p.qgrp_ctr[trow * ng + g], 1) == 32 / OUTS - 1;
            last = __shfl_sync(0xffffffffu, last, 0);
            if (last) {
                __threadfence();
                xquant_group(__ldcg(hrow + 32 * g + lane), lane, g, f, qrow);
                if (lane == 0) p.qgrp_ctr[trow * ng + g] = 0;
            }
        }
    }
}

// The reduction of job j (all CW warps' partials are in its slot): adds the
// K slices in a fixed order and writes the outputs (split parts: publishes
// them, the last part finishes); frees the slot.  Run by one warp.
template <int M, int NTK, int RTILES>
__device__ __forceinline__ void imma_reduce(const GemvParams& p, const ImmaConfig& cfg, const ImmaRedJob& j,
                                            const ImmaRed& R, int n_active, int NKS, int lane) {
    constexpr int RT = kImmaRows / M;
    constexpr int OUTS = RTILES * RT;          // outputs per item and token
    const int sq = j.r % kImmaRedSlots;
    const float* red = R.buf + (size_t)sq * R.floats;
    const int nsplit = j.seg ? cfg.seg[1].nsplit : cfg.seg[0].nsplit;
    __threadfence_block();
    bool split_done = false;
    if (nsplit == 1) {
        for (int o = lane; o < NTK * OUTS; o += 32) {
            const int q = o / OUTS, rem = o - q * OUTS;
            const int rtt = rem / RT, rr = rem - rtt * RT;
            if (q < j.nt) {
                float v[M];
#pragma unroll
                for (int m = 0; m < M; m++) {
                    float sum = 0.f;
                    for (int k2 = 0; k2 < NKS; k2++) sum += red[((k2 * RTILES + rtt) * NTK + q) * 16 + m * RT + rr];
                    v[m] = sum;
                }
                const float res = M == 2 ? swiglu(v[0], v[M - 1], p.limit) : v[0];
                const int tk = j.t0 + q;
                float* orow = j.shared ? p.out_shared + (size_t)tk * p.rows : p.out_routed + (size_t)(j.off + tk) * p.rows;
                orow[(j.tile * RTILES + rtt) * RT + rr] = res;
            }
        }
    } else {
        // split item (only the shared expert's items are split; rows = its
        // tokens): publish this part's sums; the last part of the item adds
        // the parts in order and finishes the outputs
        const int PR = p.part_rows, grow0 = j.t0;
        for (int o = lane; o < NTK * OUTS; o += 32) {
            const int q = o / OUTS, rem = o - q * OUTS;
            const int rtt = rem / RT, rr = rem - rtt * RT;
            if (q < j.nt) {
                const int col = (j.tile * RTILES + rtt) * RT + rr;
#pragma unroll
                for (int m = 0; m < M; m++) {
                    float sum = 0.f;
                    for (int k2 = 0; k2 < NKS; k2++) sum += red[((k2 * RTILES + rtt) * NTK + q) * 16 + m * RT + rr];
                    p.part_buf[(((size_t)j.part * PR + grow0 + q) * M + m) * p.rows + col] = sum;
                }
            }
        }
        __threadfence();
        __syncwarp();
        int done = 0;
        if (lane == 0) done = atomicAdd(&p.part_ctr[grow0 * p.tiles + j.tile], 1) == nsplit - 1;
        done = __shfl_sync(0xffffffffu, done, 0);
        split_done = done != 0;
        if (done) {
            __threadfence();
            for (int o = lane; o < NTK * OUTS; o += 32) {
                const int q = o / OUTS, rem = o - q * OUTS;
                const int rtt = rem / RT, rr = rem - rtt * RT;
                if (q < j.nt) {
                    const int col = (j.tile * RTILES + rtt) * RT + rr;
                    float v[M];
#pragma unroll
                    for (int m = 0; m < M; m++) {
                        float sum = 0.f;
                        for (int pp = 0; pp < nsplit; pp++)
                            sum += __ldcg(p.part_buf + (((size_t)pp * PR + grow0 + q) * M + m) * p.rows + col);
                        v[m] = sum;
                    }
                    const float res = M == 2 ? swiglu(v[0], v[M - 1], p.limit) : v[0];
                    const int tk = j.t0 + q;
                    float* orow = j.shared ? p.out_shared + (size_t)tk * p.rows : p.out_routed + (size_t)(j.off + tk) * p.rows;
                    orow[col] = res;
                }
            }
            if (lane == 0) p.part_ctr[grow0 * p.tiles + j.tile] = 0;
        }
    }
    if (M == 2 && p.qtab && (nsplit == 1 || split_done)) imma_qgroups<OUTS>(p, j, lane);
    if (M == 1 && p.fuse_combine && j.final_pass && (nsplit == 1 || split_done))
        imma_combine_tile<OUTS>(p, j.tile, n_active, lane);
    else if (p.fuse_combine)
        __threadfence();   // outputs of an earlier pass, for the tile's combiner
    __syncwarp();
    if (lane == 0) {
        R.arr[sq] = 0;
        __threadfence_block();
        *reinterpret_cast<volatile int*>(&R.tick[sq]) = j.r / kImmaRedSlots + 1;
    }
}

// Runs this warp's pending reduction once all warps' partials are in (a
// bounded wait; usually they already are).
template <int M, int NTK, int RTILES>
__device__ __forceinline__ bool imma_flush(const GemvParams& p, const ImmaConfig& cfg, ImmaRedJob& pend,
                                           const ImmaRed& R, int n_active, int NKS, int lane, volatile int* abort_flag,
                                           int32_t* err) {
    if (pend.r < 0) return true;
    if (!warp_spin_eq(&R.arr[pend.r % kImmaRedSlots], NKS * RTILES, abort_flag, err)) return false;
    imma_reduce<M, NTK, RTILES>(p, cfg, pend, R, n_active, NKS, lane);
    pend.r = -1;
    return true;
}

// Consumers: one item.  The stage is released as soon as this warp's MMAs of
// the item's last pass are done; the partials go to a reduction slot.
// Reduction r is run by warp r % CW, one reduction later (pend), so the
// reductions spread over the warps and no warp falls behind the others.
// Returns false when a wait gave up (the warp leaves).
template <int FMT, int M, int NTK, int RTILES>
__device__ __forceinline__ bool imma_item(const GemvParams& p, const ImmaConfig& cfg, const ImmaSeg g, const int* h,
                                          uint8_t* st, uint64_t* empty_bar, uint8_t* ism, int n_active, int warp,
                                          int lane, int NKS, int sb0, int sb1, const uint32_t (&bm)[4], int& rseq,
                                          ImmaRedJob& pend, const ImmaRed& R, volatile int* abort_flag, int32_t* err) {
    const int CW = NKS * RTILES;
    const int K = p.cols;
    const int gid = lane >> 2, t = lane & 3;
    const int rt = warp % RTILES;
    // the header is gone once the stage is released: keep what is needed
    const int seg = h[7], slot = h[1], off = h[3], n_tok = h[4], part = h[8], tile = h[9], tr0 = h[10], tr1 = h[11];
    const bool shared = slot >= n_active;
    const int nsbp = g.nsbp;                                 // super-blocks of this part
    const uint32_t st_u = smem_u32(st);
    const uint32_t r0 = st_u + g.field_off[0] + (rt * kImmaRows + gid) * g.pitch[0];
    const uint32_t d0 = st_u + g.field_off[1] + (rt * kImmaRows + gid) * g.pitch[1];
    const uint32_t res_u = smem_u32(ism + kImmaDataOff);
    const int res_bytes = cfg.res_rows * cfg.xtab_bytes;
    if (n_tok <= 0) {
        __syncwarp();
        if (lane == 0) mbar_arrive(empty_bar);
        return true;
    }
    for (int t0 = 0; t0 < n_tok; t0 += NTK) {
        const int nt = min(NTK, n_tok - t0);
        const bool final_pass = t0 + NTK >= n_tok;
        int trow[NTK];
#pragma unroll
        for (int q = 0; q < NTK; q++) {
            const int tk = t0 + min(q, nt - 1);
            if (t0 == 0) trow[q] = min(q, nt - 1) == 0 ? tr0 : tr1;
            else if (shared) trow[q] = p.xtab_shared_base + tk;
            else if (p.routed_by_token) trow[q] = p.pos_tok[off + tk];
            else trow[q] = off + tk;
        }
        float y[NTK][2];
        if (res_bytes > 0 || t0 == 0) {
            uint32_t tq[NTK];
#pragma unroll
            for (int q = 0; q < NTK; q++)
                tq[q] = res_bytes > 0 ? res_u + trow[q] * cfg.xtab_bytes
                                      : st_u + cfg.xtab_off + min(q, nt - 1) * cfg.xtab_bytes;
            imma_pass<FMT, NTK, true>(r0, g.pitch[0], d0, g.pitch[1], tq, nt, K, sb0, sb1, part * nsbp, lane, bm, y);
        } else {
            const uint8_t* tq[NTK];
#pragma unroll
            for (int q = 0; q < NTK; q++) tq[q] = p.xtab + (size_t)trow[q] * p.xtab_stride;
            imma_pass<FMT, NTK, false>(r0, g.pitch[0], d0, g.pitch[1], tq, nt, K, sb0, sb1, part * nsbp, lane, bm, y);
        }
        if (final_pass) {
            __syncwarp();
            if (lane == 0) mbar_arrive(empty_bar);   // this warp is done with the stage
        }
        // reduce over the 4 lanes of a row, publish the warp's partials
#pragma unroll
        for (int q = 0; q < NTK; q++)
#pragma unroll
            for (int hh = 0; hh < 2; hh++) {
                y[q][hh] += __shfl_xor_sync(0xffffffffu, y[q][hh], 1);
                y[q][hh] += __shfl_xor_sync(0xffffffffu, y[q][hh], 2);
            }
        const int r = rseq++;
        const int sq = r % kImmaRedSlots, ticket = r / kImmaRedSlots;
        if (!warp_spin_eq(&R.tick[sq], ticket, abort_flag, err)) return false;
        float* red = R.buf + (size_t)sq * R.floats;
        if (t == 0) {
#pragma unroll
            for (int q = 0; q < NTK; q++) {
                red[(warp * NTK + q) * 16 + gid] = y[q][0];
                red[(warp * NTK + q) * 16 + gid + 8] = y[q][1];
            }
        }
        __threadfence_block();
        __syncwarp();
        if (lane == 0) atomicAdd(&R.arr[sq], 1);
        // the previous reduction of this warp, then this one becomes pending
        if (!imma_flush<M, NTK, RTILES>(p, cfg, pend, R, n_active, NKS, lane, abort_flag, err)) return false;
        if (r % CW == warp) pend = ImmaRedJob{r, seg, part, tile, off, t0, nt, shared ? 1 : 0, final_pass ? 1 : 0};
    }
    return true;
}

// Registers: a sub-partition holds 16K; with 17 warps one holds 5, so a
// thread gets 96 registers, with 16 warps 128.  One-token variants run up to
// 16 consumer warps in 96 registers; two-token variants need more and run at
// most 15 (kImmaMaxWarps2).
template <int FA, int FB, int M, int NTK, int RTILES>
__global__ void __launch_bounds__(32 * ((NTK == 1 ? kImmaMaxWarps : kImmaMaxWarps2) + 1), 1)
expert_gemv_imma_kernel(GemvParams p, ImmaConfig cfg, int32_t* err) {
    static_assert(NTK >= 1 && NTK <= kImmaMaxTok, "tokens per pass");
    constexpr int ROWS = kImmaRows * RTILES;   // stage rows
    extern __shared__ __align__(128) uint8_t ism[];
    const int S = cfg.stages;
    uint64_t* full = reinterpret_cast<uint64_t*>(ism);
    uint64_t* empty = full + kTmaMaxStages;
    uint64_t* tabbar = empty + kTmaMaxStages;
    int* ctl = reinterpret_cast<int*>(ism + kImmaCtlOff);
    volatile int* abort_flag = ctl;
    int* hdr = reinterpret_cast<int*>(ism + kImmaHdrOff);     // [stage][kImmaHdrInts]
    const int res_bytes = cfg.res_rows * cfg.xtab_bytes;
    const ImmaRed R{ctl + 4, ctl + 8, reinterpret_cast<float*>(ism + kImmaDataOff + res_bytes), cfg.red_bytes / 4};
    uint8_t* data = ism + kImmaDataOff + res_bytes + kImmaRedSlots * cfg.red_bytes;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int CW = (blockDim.x >> 5) - 1;
    const int K = p.cols;

    if (tid == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], CW);
        }
        mbar_init(tabbar, 1);
        *abort_flag = 0;
        for (int q = 0; q < kImmaRedSlots; q++) R.arr[q] = R.tick[q] = 0;
        fence_barrier_init();
    }
    __syncthreads();
    // the producer of a down launch may stream weights before the predecessor
    // (gate/up) has finished; everything else waits for it
    if (p.pdl == 1 || warp != CW) pdl_wait();
    pdl_trigger();
    // the schedule of this launch (written by the router: final before a
    // down launch starts, so its producer may read it without waiting)
    const int n_active = *p.n_active;
    const int ns0 = cfg.seg[0].nsplit, ns1 = cfg.seg[1].nsplit;
    const int nA = p.mode == 2 ? 0 : n_active * p.tiles * ns0;
    const int nB = (p.mode == 1 || !p.has_shared) ? 0 : p.tiles * ns1;
    const int n_items = nA + nB;

    if (warp == CW) {
        // ---------------- producer: every lane resolves the next item (expert,
        // token run, table rows) while the current stage's copies fly; lane 0
        // waits for free stages; the lanes issue the copies in parallel
        if (p.pdl == 2 && !p.xq_a) pdl_wait();   // tables written by the predecessor
        if (lane == 0 && res_bytes > 0 && !p.xq_a) {
            mbar_arrive_expect_tx(tabbar, (uint32_t)res_bytes);
            bulk_g2s(ism + kImmaDataOff, p.xtab, (uint32_t)res_bytes, tabbar);
        }
        // the look-ahead item lives in shared memory (control area), not in
        // registers that the consumers' code would have to give up
        struct Item { int seg, slot, tile, part, e, off, n_tok, tr0, tr1; };
        Item* nxt = reinterpret_cast<Item*>(ism + kImmaCtlOff + 48);
        auto resolve = [&](int item, Item& in) {
            if (item < nA) {
                in.seg = 0;
                in.slot = item / (p.tiles * ns0);
                const int r = item - in.slot * p.tiles * ns0;
                in.tile = r / ns0;
                in.part = r - in.tile * ns0;
            } else {
                in.seg = 1;
                in.slot = n_active;
                const int j = item - nA;
                in.tile = j / ns1;
                in.part = j - in.tile * ns1;
            }
            int tok0 = -1;
            if (p.slot_info && in.seg == 0) {
                // one load: expert, first position, tokens, first token
                const int4 si = p.slot_info[in.slot];
                in.e = si.x; in.off = si.y; in.n_tok = si.z; tok0 = si.w;
            } else {
                in.e = p.active[in.slot];
                in.off = 0;
                in.n_tok = p.T;
                if (in.seg == 0) { in.off = p.offsets[in.e]; in.n_tok = p.offsets[in.e + 1] - in.off; }
            }
            // table rows of the first pass's tokens, so consumers need no global load
            const int t1 = min(1, in.n_tok - 1);
            if (in.seg == 1) { in.tr0 = p.xtab_shared_base; in.tr1 = p.xtab_shared_base + t1; }
            else if (p.routed_by_token) {
                in.tr0 = tok0 >= 0 ? tok0 : p.pos_tok[in.off];
                in.tr1 = t1 ? p.pos_tok[in.off + t1] : in.tr0;
            } else { in.tr0 = in.off; in.tr1 = in.off + t1; }
        };
        if (lane == 0 && (int)blockIdx.x < n_items) resolve(blockIdx.x, *nxt);
        __syncwarp();
        bool ok = true;
        int issued = 0;
        for (int it = 0;; it++) {
            const int s = it % S;
            const uint32_t ph = (uint32_t)(it / S) & 1u;
            if (it >= S) {
                const bool w = lane == 0 ? mbar_wait_abort(&empty[s], ph ^ 1u, abort_flag) : true;
                if (!__shfl_sync(0xffffffffu, (int)w, 0)) { ok = false; break; }
            }
            const int item = blockIdx.x + it * gridDim.x;
            int* h = hdr + s * kImmaHdrInts;
            if (item >= n_items) {
                if (lane == 0) {
                    h[0] = item;
                    mbar_arrive(&full[s]);
                }
                break;
            }
            const Item cur = *nxt;
            __syncwarp();
            const ImmaSeg g = cur.seg ? cfg.seg[1] : cfg.seg[0];
            const int ntab = res_bytes > 0 ? 0 : min(NTK, cur.n_tok);
            uint8_t* st = data + (size_t)s * cfg.stage_bytes;
            if (lane == 0) {
                h[0] = item; h[1] = cur.slot; h[2] = cur.e; h[3] = cur.off; h[4] = cur.n_tok;
                h[7] = cur.seg; h[8] = cur.part; h[9] = cur.tile; h[10] = cur.tr0; h[11] = cur.tr1;
                const uint32_t bytes = (uint32_t)(ROWS * (g.part_bytes[0] + g.part_bytes[1]) + ntab * cfg.xtab_bytes);
                mbar_arrive_expect_tx(&full[s], bytes);
            }
            __syncwarp();
            const MatDev* md = p.mats + (size_t)cur.e * 3;
            if (cur.seg == 0) imma_issue<FA, M, RTILES>(p, g, md, cur.tile, cur.part, st, &full[s], lane);
            else imma_issue<FB, M, RTILES>(p, g, md, cur.tile, cur.part, st, &full[s], lane);
            for (int q = lane; q < ntab; q += 32) {
                int trow;
                if (cur.seg == 1) trow = p.xtab_shared_base + q;
                else if (p.routed_by_token) trow = p.pos_tok[cur.off + q];
                else trow = cur.off + q;
                bulk_g2s(st + cfg.xtab_off + q * cfg.xtab_bytes, p.xtab + (size_t)trow * p.xtab_stride,
                         (uint32_t)cfg.xtab_bytes, &full[s]);
            }
            issued = it + 1;
            if (lane == 0 && item + (int)gridDim.x < n_items) resolve(item + gridDim.x, *nxt);
            __syncwarp();
        }
        if (lane == 0) {
            if (!ok) {
                *abort_flag = 1;
                atomicOr(err, (int)ERR_TIMEOUT);
                // the stages this warp filled must land before the CTA exits
                for (int it = max(0, issued - S); it < issued; it++) mbar_wait(&full[it % S], (uint32_t)(it / S) & 1u);
            }
            if (res_bytes > 0 && !p.xq_a) mbar_wait(tabbar, 0u);
        }
        return;
    }

    // ---------------- consumers
    const int gid = lane >> 2;
    const int NKS = CW / RTILES, ks = warp / RTILES;
    // this warp's K slice of a part, per segment
    const int s0a = ks * cfg.seg[0].nsbp / NKS, s0b = (ks + 1) * cfg.seg[0].nsbp / NKS;
    const int s1a = ks * cfg.seg[1].nsbp / NKS, s1b = (ks + 1) * cfg.seg[1].nsbp / NKS;
    uint32_t bm[4];   // B column pair (2j, 2j+1) of group j: lanes gid = 2j, 2j+1 supply it
#pragma unroll
    for (int g4 = 0; g4 < 4; g4++) bm[g4] = (gid >> 1) == g4 ? 0xFFFFFFFFu : 0u;
    if (res_bytes > 0 && p.xq_a) {
        // quantise the resident tables here from the f32 rows (rows < xq_split
        // from xq_a, the rest from xq_b) while the first stages stream in; no
        // consumer leaves before this barrier.  One float4 per lane covers four
        // groups; each warp issues up to 8 such loads before it quantises any.
        const int quads = K / 128, total = cfg.res_rows * quads;
        for (int base = warp; base < total; base += 8 * CW) {
            float4 v[8];
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const int w = base + u * CW;
                if (w < total) {
                    const int r = w / quads, c = w - r * quads;
                    const float* src = r < p.xq_split ? p.xq_a + (size_t)r * K : p.xq_b + (size_t)(r - p.xq_split) * K;
                    v[u] = __ldcg(reinterpret_cast<const float4*>(src) + 32 * c + lane);
                }
            }
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const int w = base + u * CW;
                if (w < total) {
                    const int r = w / quads, c = w - r * quads;
                    xquant_quad(v[u], lane, c, K, ism + kImmaDataOff + r * cfg.xtab_bytes);
                }
            }
        }
        named_barrier(1, CW * 32);
    } else if (res_bytes > 0 && !warp_wait(tabbar, 0u, abort_flag, err)) {
        return;
    }
    int rseq = 0;   // reductions this warp has taken part in (the same for every warp)
    ImmaRedJob pend;
    pend.r = -1;
    for (int it = 0;; it++) {
        const int s = it % S;
        const uint32_t ph = (uint32_t)(it / S) & 1u;
        if (!warp_wait(&full[s], ph, abort_flag, err)) return;
        const int* h = hdr + s * kImmaHdrInts;
        if (h[0] >= n_items) break;
        uint8_t* st = data + (size_t)s * cfg.stage_bytes;
        const bool ok = h[7] == 0
            ? imma_item<FA, M, NTK, RTILES>(p, cfg, cfg.seg[0], h, st, &empty[s], ism, n_active, warp, lane, NKS, s0a, s0b, bm,
                                            rseq, pend, R, abort_flag, err)
            : imma_item<FB, M, NTK, RTILES>(p, cfg, cfg.seg[1], h, st, &empty[s], ism, n_active, warp, lane, NKS, s1a, s1b, bm,
                                            rseq, pend, R, abort_flag, err);
        if (!ok) return;
    }
    imma_flush<M, NTK, RTILES>(p, cfg, pend, R, n_active, NKS, lane, abort_flag, err);
}

}  // namespace qrm
