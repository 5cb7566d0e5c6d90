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
// Per token: hi[K] int8 | lo[K] uint8 | scale[K/32] f32 | sum[K/32] f32 (sum of
// the original f32 values of the group, for the Q4_K min term).
struct XTab {
    int8_t* hi;
    uint8_t* lo;
    float* sc;
    float* sum;
};
__host__ __device__ inline int xtab_bytes(int K) { return 2 * K + 8 * (K / 32); }
__device__ __forceinline__ XTab xtab_at(uint8_t* base, int K) {
    XTab t;
    t.hi = reinterpret_cast<int8_t*>(base);
    t.lo = base + K;
    t.sc = reinterpret_cast<float*>(base + 2 * K);
    t.sum = t.sc + K / 32;
    return t;
}

// Quantises activation rows into tables (global memory), one warp per
// 32-element group.  rows: src row r -> table row r.
__global__ void xquant_kernel(const float* __restrict__ src, int K, int rows, uint8_t* __restrict__ tab,
                              int stride) {
    const int lane = threadIdx.x & 31;
    const int groups = K / 32;
    const long long total = (long long)rows * groups;
    for (long long w = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5; w < total;
         w += ((long long)gridDim.x * blockDim.x) >> 5) {
        const int r = (int)(w / groups), gi = (int)(w - (long long)r * groups);
        const float v = src[(size_t)r * K + gi * 32 + lane];
        float amax = fabsf(v), sum = v;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
            sum += __shfl_xor_sync(0xffffffffu, sum, o);
        }
        const float s = amax > 0.f ? amax * (1.f / 32767.f) : 0.f;
        int q = amax > 0.f ? __float2int_rn(v / s) : 0;
        q = max(-32767, min(32767, q));
        XTab t = xtab_at(tab + (size_t)r * stride, K);
        t.hi[gi * 32 + lane] = (int8_t)(q >> 8);          // arithmetic shift: floor(q / 256)
        t.lo[gi * 32 + lane] = (uint8_t)(q & 0xFF);       // q = 256*hi + lo
        if (lane == 0) {
            t.sc[gi] = s;
            t.sum[gi] = sum;
        }
    }
}
inline int xtab_stride(int K) { return (xtab_bytes(K) + 15) / 16 * 16; }

// ------------------------------------------------------------ formats

template <int FMT> struct ImmaFmt;

// Q4_K: 144-byte blocks (d, dmin, scales[12], qs[128]); group s of a block =
// nibble (s & 1) of qs bytes [32*(s>>1), +32).  Thread t takes bytes
// [8t, 8t+8) of the group: K slots 4t..4t+3 <- bytes 8t..8t+3, slots
// 16+4t.. <- bytes 8t+4..8t+7; the activation table uses the same order.
template <> struct ImmaFmt<Q4_K> {
    static constexpr int kBS = 256;          // weights per super-block / block
    static constexpr bool kSigned = false;   // codes are u8
    static constexpr int kFields = 1;
    __host__ __device__ static int len(int) { return 144; }
    __host__ __device__ static long long base_mul(int) { return 0; }
    // A fragments of the 8 groups of block b for rows g (r0) and g+8 (r1).
    struct Rows {
        const uint8_t* r0;
        const uint8_t* r1;
    };
    __device__ __forceinline__ static void afrag(const Rows& rw, int b, int s, int t, uint32_t (&a)[4]) {
        const int off = 144 * b + 16 + 32 * (s >> 1) + 8 * t;
        const uint2 w0 = *reinterpret_cast<const uint2*>(rw.r0 + off);
        const uint2 w1 = *reinterpret_cast<const uint2*>(rw.r1 + off);
        const int sh = 4 * (s & 1);
        a[0] = (w0.x >> sh) & 0x0F0F0F0Fu;
        a[1] = (w1.x >> sh) & 0x0F0F0F0Fu;
        a[2] = (w0.y >> sh) & 0x0F0F0F0Fu;
        a[3] = (w1.y >> sh) & 0x0F0F0F0Fu;
    }
    // scale a and min mm of (row, groups 2t and 2t+1) of block b
    __device__ __forceinline__ static void scales(const uint8_t* row, int b, int t, float (&a)[2], float (&mm)[2]) {
        const uint4 hdr = *reinterpret_cast<const uint4*>(row + 144 * b);
        const float d = h2f((uint16_t)(hdr.x & 0xFFFF)), dmin = h2f((uint16_t)(hdr.x >> 16));
        const int o = 2 * (t & 1);
        const bool high = t >= 2;
#pragma unroll
        for (int i = 0; i < 2; i++) {
            // GetScaleMinK4 (BlockDequantizer.cs:155-166) for sub-block 2t + i
            const uint32_t B0 = (hdr.y >> (8 * (o + i))) & 0xFF;
            const uint32_t B1 = (hdr.z >> (8 * (o + i))) & 0xFF;
            const uint32_t B2 = (hdr.w >> (8 * (o + i))) & 0xFF;
            const uint32_t sc = high ? ((B2 & 0xF) | ((B0 >> 6) << 4)) : (B0 & 63);
            const uint32_t m = high ? ((B2 >> 4) | ((B1 >> 6) << 4)) : (B1 & 63);
            a[i] = d * magic_int(sc);
            mm[i] = dmin * magic_int(m);
        }
    }
};

// Q8_0 (split layout): qs[nb][32] | d[nb]; group = block of 32 int8 codes.
// Stage rows: qs row pitch P, then the d rows at d_off with pitch Pd.
template <> struct ImmaFmt<Q8_0> {
    static constexpr int kBS = 32;
    static constexpr bool kSigned = true;
    static constexpr int kFields = 2;
    __host__ __device__ static int len(int f) { return f == 0 ? 32 : 2; }
    __host__ __device__ static long long base_mul(int f) { return f == 0 ? 0 : 32; }
};

// Q4_0 (split layout): qs[nb][16] | d[nb] | pad; group = block of 32 nibbles,
// low nibble of byte i = weight i, high nibble = weight 16+i, y = d*(q-8).
template <> struct ImmaFmt<Q4_0> {
    static constexpr int kBS = 32;
    static constexpr bool kSigned = false;
    static constexpr int kFields = 2;
    __host__ __device__ static int len(int f) { return f == 0 ? 16 : 2; }
    __host__ __device__ static long long base_mul(int f) { return f == 0 ? 0 : 16; }
};

// ------------------------------------------------------------ stage plan

constexpr int kImmaRows = 16;                 // MMA rows per row tile
constexpr int kImmaMaxTok = 2;                // most tokens per pass (tables in the stage)
constexpr int kImmaHdrInts = 8;               // per-stage header: item, slot, e, off, n_tok
constexpr int kImmaHdrOff = kTmaRedOff;       // [kTmaMaxStages][kImmaHdrInts] ints
constexpr int kImmaCtlOff = kImmaHdrOff + kTmaMaxStages * kImmaHdrInts * 4;
constexpr int kImmaRedOff = kTmaDataOff;      // [16 warps][NTK][32] floats
static_assert(kImmaCtlOff + 16 <= kTmaDataOff, "imma header area");
constexpr int kImmaDataOff = kImmaRedOff + 16 * kImmaMaxTok * 32 * 4;

struct ImmaConfig {
    int stages;
    int stage_bytes;     // weights + tables
    int pitch[2];        // bytes between rows of field 0 / field 1
    int field_off[2];    // offset of field f's row 0 inside a stage
    int row_bytes[2];    // bytes copied per row of field f
    int xtab_off;        // offset of the activation tables inside a stage
    int xtab_bytes;      // per token (16-byte multiple)
};

template <int FMT>
__host__ inline bool imma_plan(int cols, int rows_per_item, int ntok, int smem_budget, ImmaConfig* c) {
    using F = ImmaFmt<FMT>;
    if (cols % 256) return false;                 // super-blocks of 256 weights
    const int bpr = cols / F::kBS;
    int off = 0;
    for (int f = 0; f < F::kFields; f++) {
        const int rb = bpr * F::len(f);
        if (rb % 16) return false;
        c->row_bytes[f] = rb;
        c->pitch[f] = rb + 16;
        c->field_off[f] = off;
        off += rows_per_item * c->pitch[f];
    }
    c->xtab_off = off;
    c->xtab_bytes = xtab_stride(cols);
    off += ntok * c->xtab_bytes;
    c->stage_bytes = off;
    int s = (smem_budget - kImmaDataOff) / off;
    if (s > kTmaMaxStages) s = kTmaMaxStages;
    if (s < 2) return false;
    c->stages = s;
    return true;
}
inline size_t imma_smem_bytes(const ImmaConfig& c) { return (size_t)kImmaDataOff + (size_t)c.stages * c.stage_bytes; }

// ------------------------------------------------------------ kernel
// Item = (slot, tile) with RTILES row tiles of 16 MMA rows.  gate/up (M = 2):
// a row tile is 8 rows of gate and the same 8 rows of up (a thread holds gate
// row g and up row g); down (M = 1): 16 consecutive rows.  cw consumer warps
// (blockDim/32 - 1, chosen so the K slices are even): warp w takes row tile
// w % RTILES and K slice w / RTILES.  The producer warp resolves each item
// (expert, token run, activation rows), copies the weight rows and the
// activation tables of the first NTK tokens into the stage, and writes the
// item header, S stages ahead of the consumers.
template <int FMT, int M, int NTK, int RTILES>
__global__ void __launch_bounds__(544, 1)
expert_gemv_imma_kernel(GemvParams p, ImmaConfig cfg, int32_t* err) {
    using F = ImmaFmt<FMT>;
    static_assert(NTK >= 1 && NTK <= kImmaMaxTok, "tokens per pass");
    constexpr int RT = kImmaRows / M;          // matrix rows per row tile
    constexpr int ROWS = kImmaRows * RTILES;   // stage rows
    extern __shared__ __align__(128) uint8_t ism[];
    const int S = cfg.stages;
    uint64_t* full = reinterpret_cast<uint64_t*>(ism);
    uint64_t* empty = full + kTmaMaxStages;
    int* hdr = reinterpret_cast<int*>(ism + kImmaHdrOff);          // [stage][kImmaHdrInts]
    int* ctl = reinterpret_cast<int*>(ism + kImmaCtlOff);          // consumer broadcast
    float* red = reinterpret_cast<float*>(ism + kImmaRedOff);      // [cw][NTK][32]
    uint8_t* data = ism + kImmaDataOff;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int CW = (blockDim.x >> 5) - 1;
    const int NKS = CW / RTILES;
    const int ncons = CW * 32;
    const int K = p.cols;
    const int nsb = K / 256;
    const int n_active = *p.n_active;
    const int n_items = p.mode == 2 ? (p.has_shared ? p.tiles : 0)
                                    : (n_active + (p.mode == 0 && p.has_shared ? 1 : 0)) * p.tiles;
    const int slot_base = p.mode == 2 ? n_active : 0;

    if (tid == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], CW);
        }
        fence_barrier_init();
    }
    __syncthreads();

    if (warp == CW) {
        // ---------------- producer
        if (lane == 0) {
            bool ok = true;
            int issued = 0;
            for (int it = 0;; it++) {
                const int s = it % S;
                const uint32_t ph = (uint32_t)(it / S) & 1u;
                if (it >= S && !mbar_wait(&empty[s], ph ^ 1u)) { ok = false; break; }
                const int item = blockIdx.x + it * gridDim.x;
                int* h = hdr + s * kImmaHdrInts;
                h[0] = item;
                if (item >= n_items) { mbar_arrive(&full[s]); break; }
                const int sl = item / p.tiles, tile = item - sl * p.tiles;
                const int slot = slot_base + sl;
                const int e = p.active[slot];
                const bool shared = slot >= n_active;
                int off = 0, n_tok = p.T;
                if (!shared) { off = p.offsets[e]; n_tok = p.offsets[e + 1] - off; }
                h[1] = slot; h[2] = e; h[3] = off; h[4] = n_tok;
                const MatDev* md = p.mats + (size_t)e * 3;
                const int ntab = min(NTK, n_tok);
                uint32_t bytes = (uint32_t)(ROWS * (cfg.row_bytes[0] + (F::kFields > 1 ? cfg.row_bytes[1] : 0)) +
                                            ntab * cfg.xtab_bytes);
                mbar_arrive_expect_tx(&full[s], bytes);
                uint8_t* st = data + (size_t)s * cfg.stage_bytes;
                for (int r = 0; r < ROWS; r++) {
                    const int rt = r / kImmaRows, rr = r % kImmaRows;
                    const int m = M == 2 ? rr / RT : 0;
                    const MatDev mat = md[M == 2 ? m : 2];
                    const int row = (tile * RTILES + rt) * RT + (rr % RT);
                    for (int f = 0; f < F::kFields; f++) {
                        const uint8_t* src = mat.base + mat.nb * F::base_mul(f) + (size_t)row * cfg.row_bytes[f];
                        bulk_g2s(st + cfg.field_off[f] + r * cfg.pitch[f], src, (uint32_t)cfg.row_bytes[f], &full[s]);
                    }
                }
                for (int q = 0; q < ntab; q++) {
                    int trow;
                    if (shared) trow = p.xtab_shared_base + q;
                    else if (p.routed_by_token) trow = p.perm[off + q] / p.k;
                    else trow = off + q;
                    bulk_g2s(st + cfg.xtab_off + q * cfg.xtab_bytes, p.xtab + (size_t)trow * p.xtab_stride,
                             (uint32_t)cfg.xtab_bytes, &full[s]);
                }
                issued = it + 1;
            }
            if (!ok) {
                atomicOr(err, (int)ERR_TIMEOUT);
                for (int it = max(0, issued - S); it < issued; it++) mbar_wait(&full[it % S], (uint32_t)(it / S) & 1u);
            }
        }
        return;
    }

    // ---------------- consumers
    const int gid = lane >> 2, t = lane & 3;
    const int rt = warp % RTILES, ks = warp / RTILES;
    const int sb0 = ks * nsb / NKS, sb1 = (ks + 1) * nsb / NKS;
    // prmt selectors placing scale byte (2(t&1) + i) of a packed word at bits 16..23
    const uint32_t sel0 = 0x7044u | ((uint32_t)(2 * (t & 1)) << 8), sel1 = sel0 + 0x100u;
    // one thread does the bounded wait of each stage so every consumer takes the
    // same decision; the broadcast shares the barrier that closes the previous item
    if (tid == 0) {
        const bool ok = mbar_wait(&full[0], 0u);
        if (!ok) atomicOr(err, (int)ERR_TIMEOUT);
        ctl[0] = ok ? hdr[0] : -1;
    }
    named_barrier(1, ncons);
    for (int it = 0;; it++) {
        const int s = it % S;
        const uint32_t ph = (uint32_t)(it / S) & 1u;
        // double-buffered: thread 0 writes the next item's slot while others read this one
        const int item = ctl[it & 1];
        if (item < 0 || item >= n_items) break;
        mbar_wait(&full[s], ph);
        uint8_t* st = data + (size_t)s * cfg.stage_bytes;
        const int* h = hdr + s * kImmaHdrInts;
        const int slot = h[1], off = h[3], n_tok = h[4];
        const bool shared = slot >= n_active;
        const int tile = item - (item / p.tiles) * p.tiles;
        const uint8_t* r0 = st + cfg.field_off[0] + (rt * kImmaRows + gid) * cfg.pitch[0];
        const uint8_t* r1 = r0 + 8 * cfg.pitch[0];
        const int f1 = F::kFields > 1 ? 1 : 0;
        const uint8_t* d0 = st + cfg.field_off[f1] + (rt * kImmaRows + gid) * cfg.pitch[f1];
        const uint8_t* d1 = d0 + 8 * cfg.pitch[f1];
        for (int t0 = 0; t0 < n_tok; t0 += NTK) {
            const int nt = min(NTK, n_tok - t0);
            if (t0 > 0) {
                // later token passes: fetch their tables from global into the stage
                named_barrier(1, ncons);
                for (int q = 0; q < nt; q++) {
                    const int tk = t0 + q;
                    int trow;
                    if (shared) trow = p.xtab_shared_base + tk;
                    else if (p.routed_by_token) trow = p.perm[off + tk] / p.k;
                    else trow = off + tk;
                    const uint4* src = reinterpret_cast<const uint4*>(p.xtab + (size_t)trow * p.xtab_stride);
                    uint4* dst = reinterpret_cast<uint4*>(st + cfg.xtab_off + q * cfg.xtab_bytes);
                    for (int i = tid; i < cfg.xtab_bytes / 16; i += ncons) dst[i] = src[i];
                }
                named_barrier(1, ncons);
            }
            float y[NTK][2];
#pragma unroll
            for (int q = 0; q < NTK; q++) y[q][0] = y[q][1] = 0.f;
            for (int sb = sb0; sb < sb1; sb++) {
                // this lane's activation bytes for group gid of the super-block
                uint32_t xb[NTK][4];
#pragma unroll
                for (int q = 0; q < NTK; q++) {
                    const XTab xt = xtab_at(st + cfg.xtab_off + q * cfg.xtab_bytes, K);
                    const int kb = 256 * sb + 32 * gid;
                    if (q < nt) {
                        if (FMT == Q4_0) {
                            xb[q][0] = *reinterpret_cast<const uint32_t*>(xt.hi + kb + 4 * t);
                            xb[q][1] = *reinterpret_cast<const uint32_t*>(xt.hi + kb + 16 + 4 * t);
                            xb[q][2] = *reinterpret_cast<const uint32_t*>(xt.lo + kb + 4 * t);
                            xb[q][3] = *reinterpret_cast<const uint32_t*>(xt.lo + kb + 16 + 4 * t);
                        } else {
                            const uint2 hh = *reinterpret_cast<const uint2*>(xt.hi + kb + 8 * t);
                            const uint2 ll = *reinterpret_cast<const uint2*>(xt.lo + kb + 8 * t);
                            xb[q][0] = hh.x; xb[q][1] = hh.y; xb[q][2] = ll.x; xb[q][3] = ll.y;
                        }
                    } else {
                        xb[q][0] = xb[q][1] = xb[q][2] = xb[q][3] = 0u;
                    }
                }
                int dh[NTK][2][4], dl[NTK][2][4];   // two accumulator chains (even / odd groups)
#pragma unroll
                for (int q = 0; q < NTK; q++)
#pragma unroll
                    for (int c = 0; c < 2; c++)
#pragma unroll
                        for (int i = 0; i < 4; i++) dh[q][c][i] = dl[q][c][i] = 0;
#pragma unroll
                for (int pr = 0; pr < 4; pr++) {
                    // groups 2pr (low nibbles / first block) and 2pr+1
                    uint32_t A0[4], A1[4];
                    if (FMT == Q4_K) {
                        const int o = 144 * sb + 16 + 32 * pr + 8 * t;
                        const uint2 w0 = *reinterpret_cast<const uint2*>(r0 + o);
                        const uint2 w1 = *reinterpret_cast<const uint2*>(r1 + o);
                        // high nibbles stay in place (16 * q): the 1/16 goes into the scale
                        A0[0] = w0.x & 0x0F0F0F0Fu; A0[1] = w1.x & 0x0F0F0F0Fu; A0[2] = w0.y & 0x0F0F0F0Fu; A0[3] = w1.y & 0x0F0F0F0Fu;
                        A1[0] = w0.x & 0xF0F0F0F0u; A1[1] = w1.x & 0xF0F0F0F0u; A1[2] = w0.y & 0xF0F0F0F0u; A1[3] = w1.y & 0xF0F0F0F0u;
                    } else if (FMT == Q8_0) {
                        const int blk = 8 * sb + 2 * pr;
                        const uint2 a0 = *reinterpret_cast<const uint2*>(r0 + 32 * blk + 8 * t);
                        const uint2 a1 = *reinterpret_cast<const uint2*>(r1 + 32 * blk + 8 * t);
                        const uint2 b0 = *reinterpret_cast<const uint2*>(r0 + 32 * blk + 32 + 8 * t);
                        const uint2 b1 = *reinterpret_cast<const uint2*>(r1 + 32 * blk + 32 + 8 * t);
                        A0[0] = a0.x; A0[1] = a1.x; A0[2] = a0.y; A0[3] = a1.y;
                        A1[0] = b0.x; A1[1] = b1.x; A1[2] = b0.y; A1[3] = b1.y;
                    } else {  // Q4_0: byte i low nibble = weight i, high = weight 16+i
                        const int blk = 8 * sb + 2 * pr;
                        const uint32_t a0 = *reinterpret_cast<const uint32_t*>(r0 + 16 * blk + 4 * t);
                        const uint32_t a1 = *reinterpret_cast<const uint32_t*>(r1 + 16 * blk + 4 * t);
                        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(r0 + 16 * blk + 16 + 4 * t);
                        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(r1 + 16 * blk + 16 + 4 * t);
                        A0[0] = a0 & 0x0F0F0F0Fu; A0[1] = a1 & 0x0F0F0F0Fu;
                        A0[2] = (a0 >> 4) & 0x0F0F0F0Fu; A0[3] = (a1 >> 4) & 0x0F0F0F0Fu;
                        A1[0] = b0 & 0x0F0F0F0Fu; A1[1] = b1 & 0x0F0F0F0Fu;
                        A1[2] = (b0 >> 4) & 0x0F0F0F0Fu; A1[3] = (b1 >> 4) & 0x0F0F0F0Fu;
                    }
#pragma unroll
                    for (int half = 0; half < 2; half++) {
                        const int g8 = 2 * pr + half;
                        const uint32_t(&A)[4] = half ? A1 : A0;
#pragma unroll
                        for (int q = 0; q < NTK; q++) {
                            if (q < nt) {
                                // diagonal B: lanes of column g8 supply their bytes, others zero
                                const bool mine = gid == g8;
                                const uint32_t bh0 = mine ? xb[q][0] : 0u, bh1 = mine ? xb[q][1] : 0u;
                                const uint32_t bl0 = mine ? xb[q][2] : 0u, bl1 = mine ? xb[q][3] : 0u;
                                if (F::kSigned) {
                                    mma_s8s8(dh[q][half], A, bh0, bh1);
                                    mma_s8u8(dl[q][half], A, bl0, bl1);
                                } else {
                                    mma_u8s8(dh[q][half], A, bh0, bh1);
                                    mma_u8u8(dl[q][half], A, bl0, bl1);
                                }
                            }
                        }
                    }
                }
                // epilogue of the super-block: accumulator columns 2t, 2t+1 = groups 2t, 2t+1
                float ar[2][2], mr[2][2];   // [row g / g+8][group]: y = a * sum(code*x) - mm * sum(x)
                if (FMT == Q4_K) {
#pragma unroll
                    for (int rw = 0; rw < 2; rw++) {
                        const uint4 hd = *reinterpret_cast<const uint4*>((rw ? r1 : r0) + 144 * sb);
                        const float d = h2f((uint16_t)(hd.x & 0xFFFF)), dmin = h2f((uint16_t)(hd.x >> 16));
                        // GetScaleMinK4 (BlockDequantizer.cs:155-166), four 6-bit values per word:
                        // sc[0..3] = q[0..3] & 63, m[0..3] = q[4..7] & 63,
                        // sc[4..7] = (q[8..11] & 15) | (q[0..3] >> 6) << 4, m[4..7] = (q[8..11] >> 4) | (q[4..7] >> 6) << 4
                        const uint32_t SC = t < 2 ? (hd.y & 0x3F3F3F3Fu)
                                                  : ((hd.w & 0x0F0F0F0Fu) | ((hd.y >> 2) & 0x30303030u));
                        const uint32_t MN = t < 2 ? (hd.z & 0x3F3F3F3Fu)
                                                  : (((hd.w >> 4) & 0x0F0F0F0Fu) | ((hd.z >> 2) & 0x30303030u));
                        // byte b at bits 16..23 of 2.0f reads 2 + b/64: d*b = F*64d - 128d; the odd
                        // group (high nibbles, codes 16q) takes another 1/16
                        const float fs0 = __uint_as_float(prmt(SC, 0x40000000u, sel0));
                        const float fs1 = __uint_as_float(prmt(SC, 0x40000000u, sel1));
                        const float fm0 = __uint_as_float(prmt(MN, 0x40000000u, sel0));
                        const float fm1 = __uint_as_float(prmt(MN, 0x40000000u, sel1));
                        ar[rw][0] = fmaf(fs0, 64.f * d, -128.f * d);
                        ar[rw][1] = fmaf(fs1, 4.f * d, -8.f * d);
                        mr[rw][0] = fmaf(fm0, 64.f * dmin, -128.f * dmin);
                        mr[rw][1] = fmaf(fm1, 64.f * dmin, -128.f * dmin);
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < 2; i++) {
                        const int blk = 8 * sb + 2 * t + i;
                        const float dA = h2f(*reinterpret_cast<const uint16_t*>(d0 + 2 * blk));
                        const float dB = h2f(*reinterpret_cast<const uint16_t*>(d1 + 2 * blk));
                        ar[0][i] = dA; ar[1][i] = dB;
                        mr[0][i] = FMT == Q4_0 ? 8.f * dA : 0.f;
                        mr[1][i] = FMT == Q4_0 ? 8.f * dB : 0.f;
                    }
                }
#pragma unroll
                for (int q = 0; q < NTK; q++) {
                    if (q < nt) {
                        const XTab xt = xtab_at(st + cfg.xtab_off + q * cfg.xtab_bytes, K);
                        const float2 sx = *reinterpret_cast<const float2*>(xt.sc + 8 * sb + 2 * t);
                        const float2 sm = *reinterpret_cast<const float2*>(xt.sum + 8 * sb + 2 * t);
#pragma unroll
                        for (int i = 0; i < 2; i++) {
                            const float sxi = i ? sx.y : sx.x, smi = i ? sm.y : sm.x;
                            const int c0 = (dh[q][0][i] + dh[q][1][i]) * 256 + dl[q][0][i] + dl[q][1][i];
                            const int c1 = (dh[q][0][2 + i] + dh[q][1][2 + i]) * 256 + dl[q][0][2 + i] + dl[q][1][2 + i];
                            y[q][0] += ar[0][i] * ((float)c0 * sxi) - mr[0][i] * smi;
                            y[q][1] += ar[1][i] * ((float)c1 * sxi) - mr[1][i] * smi;
                        }
                    }
                }
            }
            // reduce over the 4 lanes of a row, then over the K slices (fixed order)
#pragma unroll
            for (int q = 0; q < NTK; q++)
#pragma unroll
                for (int hh = 0; hh < 2; hh++) {
                    y[q][hh] += __shfl_xor_sync(0xffffffffu, y[q][hh], 1);
                    y[q][hh] += __shfl_xor_sync(0xffffffffu, y[q][hh], 2);
                }
            if (t == 0) {
#pragma unroll
                for (int q = 0; q < NTK; q++) {
                    red[(warp * NTK + q) * 32 + gid] = y[q][0];
                    red[(warp * NTK + q) * 32 + gid + 8] = y[q][1];
                }
            }
            named_barrier(1, ncons);
            if (tid < NTK * RTILES * RT) {
                const int q = tid / (RTILES * RT), rem = tid - q * (RTILES * RT);
                const int rtt = rem / RT, rr = rem - rtt * RT;
                if (q < nt) {
                    float v[M];
#pragma unroll
                    for (int m = 0; m < M; m++) {
                        float sum = 0.f;
                        for (int k2 = 0; k2 < NKS; k2++)
                            sum += red[((k2 * RTILES + rtt) * NTK + q) * 32 + m * RT + rr];
                        v[m] = sum;
                    }
                    const float res = M == 2 ? swiglu(v[0], v[M - 1], p.limit) : v[0];
                    const int tk = t0 + q;
                    float* orow = shared ? p.out_shared + (size_t)tk * p.rows : p.out_routed + (size_t)(off + tk) * p.rows;
                    orow[(tile * RTILES + rtt) * RT + rr] = res;
                }
            }
        }
        // release the stage, then wait for the next one and broadcast it (one
        // barrier closes this item and opens the next)
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        if (tid == 0) {
            const int s2 = (it + 1) % S;
            const bool ok = mbar_wait(&full[s2], (uint32_t)((it + 1) / S) & 1u);
            if (!ok) atomicOr(err, (int)ERR_TIMEOUT);
            ctl[(it + 1) & 1] = ok ? hdr[s2 * kImmaHdrInts] : -1;
        }
        named_barrier(1, ncons);
    }
}

}  // namespace qrm
