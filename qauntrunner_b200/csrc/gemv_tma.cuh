// gemv_tma.cuh -- expert GEMV with bulk-copy (TMA) staging.
//
// Same work list and arithmetic contract as gemv.cuh (one persistent grid
// walks (expert, row tile) items; results are deterministic), but the weight
// bytes move HBM -> shared memory with cp.async.bulk issued by one producer
// warp into a ring of pipeline stages, each completed on an mbarrier, while
// the consumer warps decode from shared memory.  Many stages are in flight
// per SM, so HBM latency is hidden without holding weights in registers.
// No multicast and no clusters: every CTA reads its own tiles.
//
// Per stage: the tile's rows of every matrix of the item (gate+up, or down),
// each format field as one contiguous bulk copy (rows r0..r0+R-1 of a field
// array are contiguous in HBM).  Every wait is bounded: a wait that runs out
// sets ERR_TIMEOUT in the schedule and the CTA stops cleanly.
#pragma once
#include "common.cuh"
#include "gemv.cuh"

namespace qrm {

// ------------------------------------------------------------ PTX helpers

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait: gives up (returns false) after kWaitLimitNs of wall time.
constexpr uint64_t kWaitLimitNs = 2000000000ull;
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (;;) {
        for (int i = 0; i < 64; i++)
            if (mbar_try_wait(bar, parity)) return true;
        if (global_ns() - t0 > kWaitLimitNs) return false;
    }
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void fence_barrier_init() { asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory"); }
__device__ __forceinline__ void named_barrier(int id, int threads) {
    asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}
// byte K (< 128) of w as 2 + b/64 (byte placed in bits 16..23 of 2.0f)
template <int K>
__device__ __forceinline__ float pf(uint32_t w) {
    return __uint_as_float(prmt(w, 0x40000000u, 0x7044u | ((uint32_t)K << 8)));
}
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    float2 d;
    asm("{\n .reg .b64 ra, rb, rc, rd;\n mov.b64 ra, {%2,%3};\n mov.b64 rb, {%4,%5};\n mov.b64 rc, {%6,%7};\n"
        " fma.rn.f32x2 rd, ra, rb, rc;\n mov.b64 {%0,%1}, rd;\n}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return d;
}
// acc += (F(b0),F(b1)) * (x[o],x[o+1]) + (F(b2),F(b3)) * (x[o+2],x[o+3]); bytes < 128
#define QRM_PDOT4(w, X, o, acc)                                                                  \
    do {                                                                                         \
        (acc) = ffma2(make_float2(pf<0>(w), pf<1>(w)), make_float2((X)[(o)], (X)[(o) + 1]), (acc)); \
        (acc) = ffma2(make_float2(pf<2>(w), pf<3>(w)), make_float2((X)[(o) + 2], (X)[(o) + 3]), (acc)); \
    } while (0)

__device__ __forceinline__ float magic_int(uint32_t v) {  // exact float of an integer < 2^23
    return __uint_as_float(0x4B000000u | v) - 8388608.f;
}

// ------------------------------------------------------------ formats
// Stage layout per matrix: field arrays of the R tile rows back to back;
// Field f of the tile holds R*bpr blocks of len_f bytes.

template <int FMT> struct TileFmt;

template <> struct TileFmt<Q4_K> {
    static constexpr int kBS = 256, kFields = 1;
    __host__ __device__ static int len(int) { return 144; }
    __host__ __device__ static long long base_mul(int) { return 0; }
    static __device__ __forceinline__ float dot(const uint8_t* tile, int R, int bpr, int rr, int u, const XUnit& xu) {
        const uint8_t* blk = tile + (rr * bpr + (u >> 3)) * 144;
        const int j = u & 7;
        const uint4 hdr = *reinterpret_cast<const uint4*>(blk);
        const uint4 qs = *reinterpret_cast<const uint4*>(blk + 16 + 16 * j);
        // GetScaleMinK4 (BlockDequantizer.cs:155-166) for sub-blocks 2g, 2g+1
        const int g = j >> 1;
        uint32_t scA, mA, scB, mB;
        if (g < 2) {
            const uint32_t lo4 = hdr.y, mid4 = hdr.z;       // scales[0..4), [4..8)
            scA = (lo4 >> (16 * g)) & 63;
            scB = (lo4 >> (16 * g + 8)) & 63;
            mA = (mid4 >> (16 * g)) & 63;
            mB = (mid4 >> (16 * g + 8)) & 63;
        } else {
            const int s = 2 * g - 4;                        // 0 or 2: bytes j-4 / j of the formula
            const uint32_t q0 = hdr.y, q4 = hdr.z, q8 = hdr.w;
            uint32_t b8A = (q8 >> (8 * s)) & 0xFF, b8B = (q8 >> (8 * s + 8)) & 0xFF;
            uint32_t b0A = (q0 >> (8 * s)) & 0xFF, b0B = (q0 >> (8 * s + 8)) & 0xFF;
            uint32_t b4A = (q4 >> (8 * s)) & 0xFF, b4B = (q4 >> (8 * s + 8)) & 0xFF;
            scA = (b8A & 0xF) | ((b0A >> 6) << 4);
            mA = (b8A >> 4) | ((b4A >> 6) << 4);
            scB = (b8B & 0xF) | ((b0B >> 6) << 4);
            mB = (b8B >> 4) | ((b4B >> 6) << 4);
        }
        const float d = h2f((uint16_t)(hdr.x & 0xFFFF)), dmin = h2f((uint16_t)(hdr.x >> 16));
        float2 al = make_float2(0.f, 0.f), ah = make_float2(0.f, 0.f);
        const uint32_t q[4] = {qs.x, qs.y, qs.z, qs.w};
#pragma unroll
        for (int w = 0; w < 4; w++) {
            const uint32_t lo = q[w] & 0x0F0F0F0Fu, hi = (q[w] >> 4) & 0x0F0F0F0Fu;
            QRM_PDOT4(lo, xu.x, 4 * w, al);
            QRM_PDOT4(hi, xu.x, 16 + 4 * w, ah);
        }
        const float sxl = xu.s[0] + xu.s[1], sxh = xu.s[2] + xu.s[3];
        const float qxl = 64.f * ((al.x + al.y) - 2.f * sxl);
        const float qxh = 64.f * ((ah.x + ah.y) - 2.f * sxh);
        return d * (magic_int(scA) * qxl + magic_int(scB) * qxh) - dmin * (magic_int(mA) * sxl + magic_int(mB) * sxh);
    }
};

template <> struct TileFmt<Q4_0> {
    static constexpr int kBS = 32, kFields = 3;   // qs | d | pad; the pad bytes are never copied
    __host__ __device__ static int len(int f) { return f == 0 ? 16 : 2; }
    __host__ __device__ static long long base_mul(int f) { return f == 0 ? 0 : 16; }
    static __device__ __forceinline__ float dot(const uint8_t* tile, int R, int bpr, int rr, int u, const XUnit& xu) {
        const int bt = rr * bpr + u;
        const uint4 qs = *reinterpret_cast<const uint4*>(tile + bt * 16);
        const uint16_t dh = *reinterpret_cast<const uint16_t*>(tile + R * bpr * 16 + bt * 2);
        float2 al = make_float2(0.f, 0.f), ah = make_float2(0.f, 0.f);
        const uint32_t q[4] = {qs.x, qs.y, qs.z, qs.w};
#pragma unroll
        for (int w = 0; w < 4; w++) {
            const uint32_t lo = q[w] & 0x0F0F0F0Fu, hi = (q[w] >> 4) & 0x0F0F0F0Fu;
            QRM_PDOT4(lo, xu.x, 4 * w, al);
            QRM_PDOT4(hi, xu.x, 16 + 4 * w, ah);
        }
        const float sxl = xu.s[0] + xu.s[1], sxh = xu.s[2] + xu.s[3];
        const float qx = 64.f * ((al.x + al.y) - 2.f * sxl) + 64.f * ((ah.x + ah.y) - 2.f * sxh);
        return h2f(dh) * (qx - 8.f * (sxl + sxh));
    }
};

template <> struct TileFmt<Q8_0> {
    static constexpr int kBS = 32, kFields = 2;
    __host__ __device__ static int len(int f) { return f == 0 ? 32 : 2; }
    __host__ __device__ static long long base_mul(int f) { return f == 0 ? 0 : 32; }
    static __device__ __forceinline__ float dot(const uint8_t* tile, int R, int bpr, int rr, int u, const XUnit& xu) {
        const int bt = rr * bpr + u;
        const uint4 q0 = *reinterpret_cast<const uint4*>(tile + bt * 32);
        const uint4 q1 = *reinterpret_cast<const uint4*>(tile + bt * 32 + 16);
        const uint16_t dh = *reinterpret_cast<const uint16_t*>(tile + R * bpr * 32 + bt * 2);
        // low 7 bits of q+128 via prmt (2 + b/64), the top bit separately:
        // q = (b7 + 128*t) - 128 with t = top bit of b = q+128
        const uint32_t q[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
        float2 a = make_float2(0.f, 0.f);
        float top = 0.f;
#pragma unroll
        for (int w = 0; w < 8; w++) {
            const uint32_t b = q[w] ^ 0x80808080u;
            const uint32_t b7 = b & 0x7F7F7F7Fu;
            QRM_PDOT4(b7, xu.x, 4 * w, a);
            const uint32_t t = b & 0x80808080u;
            top += (t & 0x80u ? xu.x[4 * w] : 0.f) + (t & 0x8000u ? xu.x[4 * w + 1] : 0.f) +
                   (t & 0x800000u ? xu.x[4 * w + 2] : 0.f) + (t & 0x80000000u ? xu.x[4 * w + 3] : 0.f);
        }
        const float sx = (xu.s[0] + xu.s[1]) + (xu.s[2] + xu.s[3]);
        // sum b7*x = 64*(sum F x - 2 sx); sum q x = sum b7 x + 128*top - 128*sx
        return h2f(dh) * (64.f * ((a.x + a.y) - 2.f * sx) + 128.f * (top - sx));
    }
};

template <> struct TileFmt<Q6_K> {
    static constexpr int kBS = 256, kFields = 4;  // ql | qh | sc | d
    __host__ __device__ static int len(int f) { return f == 0 ? 128 : f == 1 ? 64 : f == 2 ? 16 : 2; }
    __host__ __device__ static long long base_mul(int f) { return f == 0 ? 0 : f == 1 ? 128 : f == 2 ? 192 : 208; }
    static __device__ __forceinline__ float dot(const uint8_t* tile, int R, int bpr, int rr, int u, const XUnit& xu) {
        const int bt = rr * bpr + (u >> 3);
        const int uu = u & 7, h = uu >> 2, l0 = 8 * (uu & 3), is = (uu & 3) >> 1;
        const int nbt = R * bpr;
        const uint8_t* ql = tile + bt * 128;
        const uint2 a = *reinterpret_cast<const uint2*>(ql + 64 * h + l0);
        const uint2 b = *reinterpret_cast<const uint2*>(ql + 64 * h + 32 + l0);
        const uint2 hb = *reinterpret_cast<const uint2*>(tile + nbt * 128 + bt * 64 + 32 * h + l0);
        const uint2 sc = *reinterpret_cast<const uint2*>(tile + nbt * 192 + bt * 16 + 8 * h);
        const uint16_t dh = *reinterpret_cast<const uint16_t*>(tile + nbt * 208 + bt * 2);
        float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
        const uint32_t A[2] = {a.x, a.y}, B[2] = {b.x, b.y}, H[2] = {hb.x, hb.y};
#pragma unroll
        for (int w = 0; w < 2; w++) {
            const uint32_t q1 = (A[w] & 0x0F0F0F0Fu) | ((H[w] & 0x03030303u) << 4);
            const uint32_t q2 = (B[w] & 0x0F0F0F0Fu) | (((H[w] >> 2) & 0x03030303u) << 4);
            const uint32_t q3 = ((A[w] >> 4) & 0x0F0F0F0Fu) | (((H[w] >> 4) & 0x03030303u) << 4);
            const uint32_t q4 = ((B[w] >> 4) & 0x0F0F0F0Fu) | (((H[w] >> 6) & 0x03030303u) << 4);
            QRM_PDOT4(q1, xu.x, 0 + 4 * w, acc[0]);
            QRM_PDOT4(q2, xu.x, 8 + 4 * w, acc[1]);
            QRM_PDOT4(q3, xu.x, 16 + 4 * w, acc[2]);
            QRM_PDOT4(q4, xu.x, 24 + 4 * w, acc[3]);
        }
        float r = 0.f;
#pragma unroll
        for (int g = 0; g < 4; g++) {
            const int byte = is + 2 * g;
            const uint32_t wd = byte < 4 ? sc.x : sc.y;
            const int s8 = (int)(int8_t)((wd >> (8 * (byte & 3))) & 0xFF);
            // sum (q-32) x = 64*sum F x - 160*sum x
            r += (float)s8 * (64.f * (acc[g].x + acc[g].y) - 160.f * xu.s[g]);
        }
        return h2f(dh) * r;
    }
};

template <> struct TileFmt<TRI> {
    static constexpr int kBS = 64, kFields = 2;   // codes | scale
    __host__ __device__ static int len(int f) { return f == 0 ? 16 : 2; }
    __host__ __device__ static long long base_mul(int f) { return f == 0 ? 0 : 16; }
    static __device__ __forceinline__ float dot(const uint8_t* tile, int R, int bpr, int rr, int u, const XUnit& xu) {
        const int bt = rr * bpr + (u >> 1);
        const uint2 c = *reinterpret_cast<const uint2*>(tile + bt * 16 + 8 * (u & 1));
        const uint16_t sh = *reinterpret_cast<const uint16_t*>(tile + R * bpr * 16 + bt * 2);
        // value (c & 1) - (c >> 1 & 1): each bit plane moved to bit 6 of its
        // byte reads as F = 2 or 3 (2 + b/64 with b = 0 or 64), so
        // sum v x = sum F0 x - sum F1 x
        float2 p = make_float2(0.f, 0.f), n = make_float2(0.f, 0.f);
        const uint32_t W[2] = {c.x, c.y};
#pragma unroll
        for (int w = 0; w < 2; w++) {
#pragma unroll
            for (int sh2 = 0; sh2 < 4; sh2++) {
                // codes of weights 16w + 4k + sh2 (k = byte) sit at bits 8k + 2*sh2
                const uint32_t b0 = (W[w] << (6 - 2 * sh2)) & 0x40404040u;
                const uint32_t b1 = (sh2 < 3 ? (W[w] << (5 - 2 * sh2)) : (W[w] >> 1)) & 0x40404040u;
                p = ffma2(make_float2(pf<0>(b0), pf<1>(b0)), make_float2(xu.x[16 * w + sh2], xu.x[16 * w + 4 + sh2]), p);
                p = ffma2(make_float2(pf<2>(b0), pf<3>(b0)), make_float2(xu.x[16 * w + 8 + sh2], xu.x[16 * w + 12 + sh2]), p);
                n = ffma2(make_float2(pf<0>(b1), pf<1>(b1)), make_float2(xu.x[16 * w + sh2], xu.x[16 * w + 4 + sh2]), n);
                n = ffma2(make_float2(pf<2>(b1), pf<3>(b1)), make_float2(xu.x[16 * w + 8 + sh2], xu.x[16 * w + 12 + sh2]), n);
            }
        }
        return h2f(sh) * ((p.x + p.y) - (n.x + n.y));
    }
};

// ------------------------------------------------------------ kernel

constexpr int kTmaMaxStages = 8;
constexpr int kTmaRedOff = 2 * kTmaMaxStages * 8;          // after the mbarriers
constexpr int kTmaRedFloats = 17 * 32;                      // [16 warps + final][32]
constexpr int kTmaItemsOff = kTmaRedOff + kTmaRedFloats * 4;
constexpr int kTmaDataOff = (kTmaItemsOff + (kTmaMaxStages + 1) * 4 + 127) / 128 * 128;

struct TmaConfig {
    int stages;
    int stage_bytes;     // data bytes of one stage
    int field_off[2][4]; // byte offset of (matrix, field) inside a stage
    int field_bytes[4];  // bytes of one field for the R tile rows
};

template <int FMT>
__host__ inline bool tma_plan(int M, int R, int cols, int smem_budget, TmaConfig* c) {
    using F = TileFmt<FMT>;
    const int bpr = cols / F::kBS;
    int off = 0;
    const int nf = FMT == Q4_0 ? 2 : F::kFields;   // Q4_0 pad bytes stay in HBM
    for (int m = 0; m < M; m++)
        for (int f = 0; f < nf; f++) {
            int b = R * bpr * F::len(f);
            if (b % 16) return false;
            c->field_bytes[f] = b;
            c->field_off[m][f] = off;
            off += b;
        }
    c->stage_bytes = off;
    int s = (smem_budget - kTmaDataOff) / off;
    if (s > kTmaMaxStages) s = kTmaMaxStages;
    if (s < 2) return false;
    c->stages = s;
    return true;
}

inline size_t tma_smem_bytes(const TmaConfig& c) { return (size_t)kTmaDataOff + (size_t)c.stages * c.stage_bytes; }

// Consumers: G groups of `cwg` warps (one thread per 32-weight unit of a
// row); group g computes the (matrix, row) pairs g, g+G, ... of the tile.
// One extra producer warp issues the bulk copies.
template <int FMT, int M, int R, int NT, int G>
__global__ void __launch_bounds__(544, 1)
expert_gemv_tma_kernel(GemvParams p, TmaConfig cfg, int32_t* err) {
    using F = TileFmt<FMT>;
    constexpr int PAIRS = M * R / G;      // (matrix, row) pairs per thread
    constexpr int NV = PAIRS * NT;
    static_assert(M * R % G == 0, "G must divide M*R");
    static_assert(NV <= 32 && (NV & (NV - 1)) == 0, "NV must be a power of two <= 32");
    extern __shared__ __align__(128) uint8_t tsmem[];
    const int S = cfg.stages;
    uint64_t* full = reinterpret_cast<uint64_t*>(tsmem);
    uint64_t* empty = full + kTmaMaxStages;
    float* red = reinterpret_cast<float*>(tsmem + kTmaRedOff);
    int* items = reinterpret_cast<int*>(tsmem + kTmaItemsOff);
    uint8_t* data = tsmem + kTmaDataOff;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int cwarps = (blockDim.x >> 5) - 1;     // consumer warps = G * cwg
    const int cwg = cwarps / G;
    const int ncons = cwarps * 32;
    const int U = p.cols >> 5;
    const int bpr = p.cols / F::kBS;
    const int n_active = *p.n_active;
    const int n_items = p.mode == 2 ? (p.has_shared ? p.tiles : 0)
                                    : (n_active + (p.mode == 0 && p.has_shared ? 1 : 0)) * p.tiles;
    const int slot_base = p.mode == 2 ? n_active : 0;
    const int nf = FMT == Q4_0 ? 2 : F::kFields;

    if (tid == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], cwarps);
        }
        fence_barrier_init();
    }
    __syncthreads();

    if (warp == cwarps) {
        // ---------------- producer
        if (lane == 0) {
            bool ok = true;
            int issued = 0;
            for (int it = 0;; it++) {
                const int s = it % S;
                const uint32_t ph = (uint32_t)(it / S) & 1u;
                if (it >= S && !mbar_wait(&empty[s], ph ^ 1u)) { ok = false; break; }
                // static striding: CTA b takes items b, b + grid, ... (consecutive items
                // are tiles of the same expert, so every CTA gets a share of each expert)
                const int item = blockIdx.x + it * gridDim.x;
                items[s] = item;
                if (item >= n_items) { mbar_arrive(&full[s]); break; }
                const int sl = item / p.tiles, tile = item - sl * p.tiles;
                const int e = p.active[slot_base + sl];
                const MatDev* md = p.mats + (size_t)e * 3;
                const int r0 = tile * R;
                mbar_arrive_expect_tx(&full[s], (uint32_t)cfg.stage_bytes);
                uint8_t* st = data + (size_t)s * cfg.stage_bytes;
#pragma unroll
                for (int m = 0; m < M; m++) {
                    const MatDev mat = md[M == 2 ? m : 2];
                    for (int f = 0; f < nf; f++) {
                        const uint8_t* src = mat.base + mat.nb * F::base_mul(f) + (size_t)r0 * bpr * F::len(f);
                        bulk_g2s(st + cfg.field_off[m][f], src, (uint32_t)cfg.field_bytes[f], &full[s]);
                    }
                }
                issued = it + 1;
            }
            if (!ok) {
                atomicOr(err, (int)ERR_TIMEOUT);
                // let the copies in flight land before the CTA exits
                for (int it = max(0, issued - S); it < issued; it++) mbar_wait(&full[it % S], (uint32_t)(it / S) & 1u);
            }
        }
        return;
    }

    // ---------------- consumers
    const int g = warp / cwg;
    const int u = tid - g * cwg * 32;
    const bool has_unit = u < U;
    int* ctl = items + kTmaMaxStages;   // consumer broadcast slot
    const int toff0 = cfg.field_off[0][0], toff1 = cfg.field_off[M - 1][0];
    const float* cur_xrow = nullptr;    // activation unit cached across items (NT == 1)
    XUnit xc;
    for (int it = 0;; it++) {
        const int s = it % S;
        const uint32_t ph = (uint32_t)(it / S) & 1u;
        // one thread does the bounded wait so that every consumer takes the
        // same decision; the others then see the completed phase at once
        if (tid == 0) {
            const bool ok = mbar_wait(&full[s], ph);
            if (!ok) atomicOr(err, (int)ERR_TIMEOUT);
            *ctl = ok ? items[s] : -1;
        }
        named_barrier(1, ncons);
        const int item = *ctl;
        if (item < 0 || item >= n_items) break;
        mbar_wait(&full[s], ph);
        const uint8_t* st = data + (size_t)s * cfg.stage_bytes;
        const int sl = item / p.tiles, tile = item - sl * p.tiles;
        const int slot = slot_base + sl;
        const int e = p.active[slot];
        const bool shared = slot >= n_active;
        const int r0 = tile * R;
        int n_tok, off = 0;
        if (shared) n_tok = p.T_sh;
        else { off = p.offsets[e]; n_tok = p.offsets[e + 1] - off; }
        for (int t0 = 0; t0 < n_tok; t0 += NT) {
            if (t0 > 0) named_barrier(1, ncons);   // red is reused by the next chunk
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
                        if (NT > 1 || xrow != cur_xrow) {
                            load_x<FMT>(xc, xrow, u);
                            cur_xrow = xrow;
                        }
#pragma unroll
                        for (int pi = 0; pi < PAIRS; pi++) {
                            const int gp = g + pi * G;
                            const int m = gp / R, rr = gp - m * R;
                            acc[pi * NT + t] = F::dot(st + (m == 0 ? toff0 : toff1), R, bpr, rr, u, xc);
                        }
                    }
                }
            }
            const float v = warp_reduce_transposed<NV>(acc, lane);
            if (transposed_writer<NV>(lane)) red[warp * 32 + transposed_index<NV>(lane)] = v;
            named_barrier(1, ncons);
            if (tid < R * NT) {
                // value (pair gp, token t) lives in group gp % G at index (gp / G) * NT + t
                const int rr = tid / NT, t = tid - rr * NT;
                if (t0 + t < n_tok) {
                    float val[M];
#pragma unroll
                    for (int m = 0; m < M; m++) {
                        const int gp = m * R + rr, gg = gp % G, li = (gp / G) * NT + t;
                        float sum = 0.f;
                        for (int wi = 0; wi < cwg; wi++) sum += red[(gg * cwg + wi) * 32 + li];
                        val[m] = sum;
                    }
                    const float res = M == 2 ? swiglu(val[0], val[M - 1], p.limit) : val[0];
                    float* orow = shared ? p.out_shared + (size_t)(t0 + t) * p.rows
                                         : p.out_routed + (size_t)(off + t0 + t) * p.rows;
                    orow[r0 + rr] = res;
                }
            }
        }
        // release the stage (one arrival per consumer warp)
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
}

}  // namespace qrm
