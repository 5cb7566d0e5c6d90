// route.cuh -- RMSNorm, router logits, top-k and dispatch.
//
// Routing must reproduce the reference bit for bit, so these kernels emulate
// the reference's float operation order exactly (no FMA contraction: every
// product and sum goes through __fmul_rn / __fadd_rn):
//  * TransformerOps.RmsNorm (TransformerOps.cs:12-40): eight lane sums
//    acc[j] over columns c = j mod 8, each a sequential chain of
//    acc + x*x, then HSum (SimdMath.cs:17-22) = ((0+acc0)+acc1)+...+acc7,
//    the tail columns, scale = 1/sqrt(ss/n + eps), out = (x*scale)*w.
//  * Router logits = SimdMath.DotF32 (SimdMath.cs:34-53) of each router row
//    with xn, the same eight-chain structure.
//  * Softmax (StreamingEngine.cs:642-647) with a sequential sum, SelectTopK
//    (801-810); GLM sigmoid + bias + SelectTopKIndices (730-767, 793-799).
// A chain of d/8 dependent adds cannot be split, so parallelism comes from
// running the T*E*8 chains side by side.
#pragma once
#include "common.cuh"
#include "gemv_tma.cuh"
#include "ep.cuh"
#include "glibc_expf.cuh"

namespace qrm {

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

// acc + sum over i = lane, lane+8, ... < n8 of a[i]*b[i], in that order (one
// Vector256 lane of SimdMath.DotF32 / RmsNorm).  The sixteen products of the
// next block are formed while the current block's dependent adds run.
__device__ __forceinline__ float lane_chain(const float* __restrict__ a, const float* __restrict__ b, int lane,
                                            int n8, float acc) {
    int i = 0;
    if (n8 >= 256) {
        // three-stage pipeline over blocks of 16 steps: the operands of block
        // i+2 are loaded and the products of block i+1 formed while block i's
        // dependent adds run, so no add waits on a load
        float ra[16], rb[16], p[16];
#pragma unroll
        for (int u = 0; u < 16; u++) p[u] = __fmul_rn(a[8 * u + lane], b[8 * u + lane]);
#pragma unroll
        for (int u = 0; u < 16; u++) { ra[u] = a[128 + 8 * u + lane]; rb[u] = b[128 + 8 * u + lane]; }
        for (i = 256; i + 128 <= n8; i += 128) {
#pragma unroll
            for (int u = 0; u < 16; u++) {
                acc = __fadd_rn(acc, p[u]);
                p[u] = __fmul_rn(ra[u], rb[u]);
                ra[u] = a[i + 8 * u + lane];
                rb[u] = b[i + 8 * u + lane];
            }
        }
#pragma unroll
        for (int u = 0; u < 16; u++) {
            acc = __fadd_rn(acc, p[u]);
            p[u] = __fmul_rn(ra[u], rb[u]);
        }
#pragma unroll
        for (int u = 0; u < 16; u++) acc = __fadd_rn(acc, p[u]);
    }
    for (; i < n8; i += 8) acc = __fadd_rn(acc, __fmul_rn(a[i + lane], b[i + lane]));
    return acc;
}

// lane_chain(a, a, ...) with one load per step: acc + sum of a[i]*a[i] over
// i = lane, lane+8, ... < n8, in that order (the RMSNorm sum of squares,
// TransformerOps.cs:18-24)
__device__ __forceinline__ float lane_chain_sq(const float* __restrict__ a, int lane, int n8, float acc) {
    int i = 0;
    if (n8 >= 256) {
        float ra[16], p[16];
#pragma unroll
        for (int u = 0; u < 16; u++) { const float v = a[8 * u + lane]; p[u] = __fmul_rn(v, v); }
#pragma unroll
        for (int u = 0; u < 16; u++) ra[u] = a[128 + 8 * u + lane];
        for (i = 256; i + 128 <= n8; i += 128) {
#pragma unroll
            for (int u = 0; u < 16; u++) {
                acc = __fadd_rn(acc, p[u]);
                p[u] = __fmul_rn(ra[u], ra[u]);
                ra[u] = a[i + 8 * u + lane];
            }
        }
#pragma unroll
        for (int u = 0; u < 16; u++) {
            acc = __fadd_rn(acc, p[u]);
            p[u] = __fmul_rn(ra[u], ra[u]);
        }
#pragma unroll
        for (int u = 0; u < 16; u++) acc = __fadd_rn(acc, p[u]);
    }
    for (; i < n8; i += 8) acc = __fadd_rn(acc, __fmul_rn(a[i + lane], a[i + lane]));
    return acc;
}

// Sequential HSum of eight lane accumulators (SimdMath.HSum).
__device__ __forceinline__ float hsum8_seq(const float* a) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 8; i++) s = __fadd_rn(s, a[i]);
    return s;
}

// ---------------------------------------------------------------------------
// Small-T router: each CTA owns EPC experts and all T tokens (T <= 8 and
// small enough for shared memory), loads the router rows and the inputs into
// shared memory with cp.async (all bytes in flight at once, one commit group
// per column chunk), recomputes the RMSNorm of its tokens in place and runs
// the T*EPC*8 logit chains.  CTA 0 also writes xn for the expert kernels.
// Shared memory: W[EPC][d] | X[T][d] (normalised in place) | red | scl.
constexpr int kSmallT = 8;
constexpr int kRouteEPC = 2;
constexpr int kRouteThreads = 128;
constexpr int kRouteChunks = 4;

struct RouteParams {
    const float* x;        // [T x d]
    const float* norm_w;   // [d] or null
    const float* router;   // [E x d]
    const float* offset;   // [E] or null
    float* xn;             // [T x d] out
    float* logits;         // [T x E] out
    int T, d, E;
    int apply_norm;
    float eps;
};

inline size_t route_small_smem(int d, int T) {
    return sizeof(float) * ((size_t)(kRouteEPC + T) * d + (size_t)T * kRouteEPC * 8 + T);
}
inline int route_small_max_tokens(int d) {
    int t = kSmallT;
    while (t > 0 && route_small_smem(d, t) > 220 * 1024) t--;
    return t;
}

template <int C>
__device__ __forceinline__ void cp_async_wait_chunk() {
    cp_async_wait<kRouteChunks - 1 - C>();
}

__global__ void __launch_bounds__(kRouteThreads)
route_small_kernel(RouteParams p) {
    extern __shared__ __align__(16) float smem[];
    const int d = p.d, T = p.T;
    const int e0 = blockIdx.x * kRouteEPC;
    const int ne = min(kRouteEPC, p.E - e0);
    float* W = smem;                        // [EPC][d]
    float* X = W + kRouteEPC * d;           // [T][d]
    float* red = X + T * d;                 // [T*EPC*8]
    float* scl = red + T * kRouteEPC * 8;   // [T]
    const int tid = threadIdx.x;
    const int d4 = d / 4;                   // d % 4 == 0 (host check)
    const int d8 = d / 8 * 8;
    const int g8 = d8 / 8;
    const int chg = (g8 + kRouteChunks - 1) / kRouteChunks;   // 8-column groups per chunk

    // issue every load now; chunk c = columns [8*c*chg, 8*(c+1)*chg), the
    // last chunk also carries the < 8 tail columns
    for (int c = 0; c < kRouteChunks; c++) {
        int lo = min(d4, 2 * c * chg);
        int hi = (c == kRouteChunks - 1) ? d4 : min(d4, 2 * (c + 1) * chg);
        int w4 = hi - lo, rows = ne + T;
        for (int i = tid; i < rows * w4; i += kRouteThreads) {
            int r = i / w4, q = lo + i % w4;
            if (r < ne) cp_async16(W + r * d + 4 * q, p.router + (size_t)(e0 + r) * d + 4 * q);
            else cp_async16(X + (r - ne) * d + 4 * q, p.x + (size_t)(r - ne) * d + 4 * q);
        }
        cp_async_commit();
    }

    // RMSNorm chains, thread (t, j) for t < T, j < 8, chunk by chunk as data lands
    const bool norm_thread = p.apply_norm && tid < T * 8;
    const int nt = tid >> 3, nj = tid & 7;
    float acc = 0.f;
#define QRM_ROUTE_CHUNK(C)                                                        \
    cp_async_wait_chunk<C>();                                                     \
    __syncthreads();                                                              \
    if (norm_thread) {                                                            \
        const float* xr = X + nt * d + 8 * (C) * chg;                             \
        int stop = min(d8, 8 * ((C) + 1) * chg) - 8 * (C) * chg;                  \
        if (stop > 0) acc = lane_chain_sq(xr, nj, stop, acc);                         \
    }
    QRM_ROUTE_CHUNK(0)
    QRM_ROUTE_CHUNK(1)
    QRM_ROUTE_CHUNK(2)
    QRM_ROUTE_CHUNK(3)
#undef QRM_ROUTE_CHUNK
    if (p.apply_norm) {
        if (norm_thread) red[nt * 8 + nj] = acc;
        __syncthreads();
        if (tid < T) {
            const float* xr = X + tid * d;
            float ss = 0.f;
            int i = 0;
            if (d >= 8) { ss = hsum8_seq(red + tid * 8); i = d8; }
            for (; i < d; i++) ss = __fadd_rn(ss, __fmul_rn(xr[i], xr[i]));
            float v = __fadd_rn(__fdiv_rn(ss, (float)d), p.eps);
            scl[tid] = __fdiv_rn(1.f, __fsqrt_rn(v));
        }
        __syncthreads();
        for (int t = 0; t < T; t++) {
            const float sc = scl[t];
            float* xr = X + t * d;
            for (int c = tid; c < d; c += kRouteThreads) {
                float v = __fmul_rn(xr[c], sc);
                if (p.norm_w) v = __fmul_rn(v, p.norm_w[c]);
                xr[c] = v;
            }
        }
        __syncthreads();
    }
    if (blockIdx.x == 0)
        for (int i = tid; i < T * d; i += kRouteThreads) p.xn[i] = X[i];

    // logit chains: thread (t, e, j)
    const int lt = tid / (kRouteEPC * 8), le = (tid >> 3) % kRouteEPC, lj = tid & 7;
    const bool lthread = lt < T && le < ne;
    if (lthread) {
        const float* wr = W + le * d;
        const float* xr = X + lt * d;
        red[(lt * kRouteEPC + le) * 8 + lj] = lane_chain(wr, xr, lj, d8, 0.f);
    }
    __syncthreads();
    if (tid < T * ne) {
        int t = tid / ne, e = tid - t * ne;
        const float* wr = W + e * d;
        const float* xr = X + t * d;
        float s = 0.f;
        int i = 0;
        if (d >= 8) { s = hsum8_seq(red + (t * kRouteEPC + e) * 8); i = d8; }
        for (; i < d; i++) s = __fadd_rn(s, __fmul_rn(wr[i], xr[i]));
        if (p.offset) s = __fadd_rn(s, p.offset[e0 + e]);
        p.logits[(size_t)t * p.E + e0 + e] = s;
    }
}

// ---------------------------------------------------------------------------
// RMSNorm of one token row per CTA (256 threads): the row and the norm
// weights are copied into shared memory with every 16-byte piece in flight
// at once, then lanes 0..7 of warp 0 run the eight chains from there (a
// chain of d/8 dependent adds fed from DRAM would wait on the memory latency
// every few steps), and all threads write the scaled row.  x 16-byte aligned,
// d % 4 == 0.
constexpr int kNormRowThreads = 256;
inline size_t rmsnorm_row_smem(int d) { return sizeof(float) * 2 * (size_t)d; }

__global__ void __launch_bounds__(kNormRowThreads) rmsnorm_row_kernel(const float* __restrict__ x,
                                                                      const float* __restrict__ w,
                                                                      float* __restrict__ xn, int d, float eps) {
    extern __shared__ __align__(16) float nrm[];   // [d] row | [d] weights
    __shared__ float sc;
    const int tid = threadIdx.x, t = blockIdx.x;
    const float* xr = x + (size_t)t * d;
    float* sw = nrm + d;
    for (int i = tid; i < d / 4; i += kNormRowThreads) {
        cp_async16(nrm + 4 * i, xr + 4 * i);
        if (w) cp_async16(sw + 4 * i, w + 4 * i);
    }
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();
    if (tid < 32) {
        const int d8 = d / 8 * 8;
        float acc = 0.f;
        if (tid < 8 && d >= 8) acc = lane_chain_sq(nrm, tid, d8, 0.f);
        float a[8];
#pragma unroll
        for (int j = 0; j < 8; j++) a[j] = __shfl_sync(0xffffffffu, acc, j);
        if (tid == 0) {
            float ss = 0.f;
            int i0 = 0;
            if (d >= 8) { ss = hsum8_seq(a); i0 = d8; }
            for (int i = i0; i < d; i++) ss = __fadd_rn(ss, __fmul_rn(nrm[i], nrm[i]));
            sc = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)d), eps)));
        }
    }
    __syncthreads();
    const float scale = sc;
    float* o = xn + (size_t)t * d;
    for (int i = tid; i < d / 4; i += kNormRowThreads) {
        float4 v = reinterpret_cast<const float4*>(nrm)[i];
        v.x = __fmul_rn(v.x, scale); v.y = __fmul_rn(v.y, scale);
        v.z = __fmul_rn(v.z, scale); v.w = __fmul_rn(v.w, scale);
        if (w) {
            const float4 g = reinterpret_cast<const float4*>(sw)[i];
            v.x = __fmul_rn(v.x, g.x); v.y = __fmul_rn(v.y, g.y);
            v.z = __fmul_rn(v.z, g.z); v.w = __fmul_rn(v.w, g.w);
        }
        reinterpret_cast<float4*>(o)[i] = v;
    }
}

// RMSNorm for any row alignment: one warp per token; lanes 0..7 run the eight
// chains straight from global memory.
__global__ void rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ w,
                               float* __restrict__ xn, int T, int d, float eps) {
    int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (warp >= T) return;
    const float* xr = x + (size_t)warp * d;
    const int d8 = d / 8 * 8;
    float acc = 0.f;
    if (lane < 8 && d >= 8) acc = lane_chain_sq(xr, lane, d8, 0.f);
    float a[8];
#pragma unroll
    for (int j = 0; j < 8; j++) a[j] = __shfl_sync(0xffffffffu, acc, j);
    float ss = 0.f;
    int i0 = 0;
    if (d >= 8) { ss = hsum8_seq(a); i0 = d8; }
    for (int i = i0; i < d; i++) ss = __fadd_rn(ss, __fmul_rn(xr[i], xr[i]));
    float scale = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)d), eps)));
    float* o = xn + (size_t)warp * d;
    for (int i = lane; i < d; i += 32) {
        float v = __fmul_rn(xr[i], scale);
        if (w) v = __fmul_rn(v, w[i]);
        o[i] = v;
    }
}

// ---------------------------------------------------------------------------
// Top-k: one warp per token.
// Ranking = Array.Sort(idx, (a, b) => v[b].CompareTo(v[a])): value
// descending, NaN last; exact ties by index ascending.
constexpr int kMaxE = 512;   // GlmMoeFfn caps n_experts at 512 (StreamingEngine.cs:733)
constexpr int kMaxK = 8;     // StreamingEngine.cs:628

struct TopkParams {
    const float* logits;      // [T x E]
    const float* bias;        // [E] or null (GLM router_bias)
    int32_t* topk_idx;        // [T x k]
    float* topk_w;            // [T x k]
    int T, E, k;
    int sigmoid;
    float routed_scale;
};

// order-preserving key of a ranking value: larger value -> larger key, NaN
// lowest, -0 == +0 (Array.Sort with v[b].CompareTo(v[a]), value descending)
__device__ __forceinline__ uint32_t rank_key(float v) {
    if (isnan(v)) return 0u;
    const uint32_t u = __float_as_uint(__fadd_rn(v, 0.f));   // -0 -> +0
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// k rounds of "largest key, then lowest index" over the candidates whose
// keys + 1 lane l holds in kc (candidate l + 32 i; 0 = none or taken): value
// descending, index ascending, a total order, by two warp reductions per
// round.  Returns the r-th winner on lane r < k.
template <int J>
__device__ __forceinline__ int warp_select(uint32_t (&kc)[J], int k, int lane) {
    int sel = -1;
#pragma unroll 1
    for (int r = 0; r < k; r++) {
        uint32_t bk = 0u;
        int bi = 0;
#pragma unroll
        for (int i = 0; i < J; i++)
            if (kc[i] > bk) { bk = kc[i]; bi = i; }   // strict: the lowest i (index) among equal keys
        const uint32_t wk = __reduce_max_sync(0xffffffffu, bk);
        const uint32_t wc = __reduce_min_sync(0xffffffffu, bk == wk ? (uint32_t)(lane + 32 * bi) : 0xffffffffu);
        const bool mine = (int)wc - 32 * bi == lane && bk == wk;   // the owner drops the winner
#pragma unroll
        for (int i = 0; i < J; i++)
            if (mine && i == bi) kc[i] = 0u;
        if (lane == r) sel = (int)wc;
    }
    return sel;
}

// Top-k of token t by one warp.  Scores (softmax: StreamingEngine.cs:642-647,
// max from float.MinValue skipping NaN, sequential sum; GLM sigmoid + bias:
// 730-767) go to the warp's shared scratch sv (weight sources) and key
// (ranking keys), E entries each; lane l then holds the keys of candidates l,
// l+32, ... in registers for the selection (SelectTopK 801-810 /
// SelectTopKIndices 793-799), and the weights are normalised in rank order
// (the sum sequential on one lane's shuffles).  Writes topk_idx / topk_w of
// token t and returns the r-th expert on lane r < k (-1 on the other lanes).
// All loads are issued first (one memory round trip); the loops over E are
// then kept rolled: this code runs once per forward, usually with its
// instructions cold in every cache, so its length costs more than its
// instruction count.  tab: the exp table in shared memory.
template <int J>
__device__ int topk_warp(const TopkParams& tp, int t, int lane, float* sv, uint32_t* key, const uint64_t* tab) {
    const int E = tp.E, k = tp.k;
    const float* lg = tp.logits + (size_t)t * E;   // read through L2: other CTAs wrote it
    {   // logits into sv, bias bits into key
        float lv[J], bv[J];
#pragma unroll
        for (int i = 0; i < J; i++) {
            const int c = lane + 32 * i;
            lv[i] = c < E ? __ldcg(lg + c) : 0.f;
            bv[i] = c < E && tp.sigmoid && tp.bias ? tp.bias[c] : 0.f;
        }
#pragma unroll
        for (int i = 0; i < J; i++) {
            const int c = lane + 32 * i;
            if (c < E) {
                sv[c] = lv[i];
                key[c] = __float_as_uint(bv[i]);
            }
        }
    }
    if (!tp.sigmoid) {
        float mx = -3.40282347e+38f;
#pragma unroll 1
        for (int i = lane; i < E; i += 32) {
            const float a = sv[i];
            if (a > mx) mx = a;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) { const float b = __shfl_xor_sync(0xffffffffu, mx, o); if (b > mx) mx = b; }
#pragma unroll 1
        for (int i = lane; i < E; i += 32) sv[i] = expf_glibc_t(__fsub_rn(sv[i], mx), tab);
        __syncwarp();
        float sum = 0.f;
        if (lane == 0) {   // sequential sum in index order
            int i = 0;
#pragma unroll 1
            for (; i + 16 <= E; i += 16) {
                float q[16];
#pragma unroll
                for (int u = 0; u < 16; u++) q[u] = sv[i + u];
#pragma unroll
                for (int u = 0; u < 16; u++) sum = __fadd_rn(sum, q[u]);
            }
#pragma unroll 1
            for (; i < E; i++) sum = __fadd_rn(sum, sv[i]);
        }
        const float inv = __fdiv_rn(1.f, __shfl_sync(0xffffffffu, sum, 0));
        __syncwarp();
#pragma unroll 1
        for (int i = lane; i < E; i += 32) {
            const float q = __fmul_rn(sv[i], inv);
            sv[i] = q;
            key[i] = rank_key(q);
        }
    } else {
#pragma unroll 1
        for (int i = lane; i < E; i += 32) {
            const float sg = __fdiv_rn(1.f, __fadd_rn(1.f, expf_glibc_t(-sv[i], tab)));
            sv[i] = sg;
            key[i] = rank_key(tp.bias ? __fadd_rn(sg, __uint_as_float(key[i])) : sg);
        }
    }
    uint32_t kc[J];
#pragma unroll
    for (int i = 0; i < J; i++) {
        const int c = lane + 32 * i;
        kc[i] = c < E ? key[c] + 1u : 0u;   // keys are below 0xFF800001: no wrap
    }
    const int e = warp_select<J>(kc, k, lane);
    const float se = lane < k ? sv[e] : 0.f;
    float sum = 0.f;
#pragma unroll 1
    for (int r = 0; r < k; r++) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, se, r));
    if (lane < k) {
        float wv;
        if (!tp.sigmoid) {
            wv = __fdiv_rn(se, sum <= 0.f ? 1.f : sum);
        } else {
            const float inv2 = __fdiv_rn(1.f, __fadd_rn(sum, 1e-20f));
            wv = __fmul_rn(__fmul_rn(se, inv2), tp.routed_scale);
        }
        tp.topk_idx[(size_t)t * k + lane] = e;
        tp.topk_w[(size_t)t * k + lane] = wv;
    }
    return e;
}

// Top-k for batches above the fused dispatch: one warp per token, 4 per CTA.
template <int J>
__global__ void __launch_bounds__(128) topk_kernel(TopkParams p) {
    __shared__ float sv[4][kMaxE];
    __shared__ uint32_t key[4][kMaxE];
    __shared__ uint64_t tab[32];
    const int wib = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x < 32) tab[lane] = kExpfTabDev[lane];
    __syncthreads();
    const int t = blockIdx.x * 4 + wib;
    if (t < p.T) topk_warp<J>(p, t, lane, sv[wib], key[wib], tab);
}

// ---------------------------------------------------------------------------
// Dispatch: stable counting sort of the T*k assignments a = t*k + j by
// expert (order inside an expert = a ascending), one CTA.  Also builds the
// work schedule of the expert kernels.
struct Schedule {
    int32_t n_active;         // routed experts (of the local window) with assignments
    int32_t err;              // device error flags (ERR_*)
    int32_t ctr[4];           // work counters: gate/up, gate/up shared, down, down shared
    int32_t route_arrivals;   // CTAs of the fused router done with their logits (0 between launches)
    int32_t pad;
};

struct DispatchParams {
    const int32_t* topk_idx;  // [T*k]
    int32_t* perm;            // [T*k]
    int32_t* inv_perm;        // [T*k]
    int32_t* pos_tok;         // [T*k] token of the assignment at each position
    int4* slot_info;          // [E+1] per active slot: expert, first position, tokens, first token
    int32_t* offsets;         // [E+1]
    int32_t* active;          // [E+1] slot -> expert (E = shared)
    Schedule* sched;
    int T, k, E;
    int first_expert, n_local;  // local expert window (EP); full range otherwise
    int has_shared;
    // expert parallelism over peer memory: wait for the records of all ep_G
    // ranks (flags reach this rank's epoch + 1), then advance the epoch
    const uint32_t* ep_flags; // [ep_G] or null
    uint32_t* ep_epoch;
    int ep_G;
    int T_sh;                 // tokens of the shared expert's slot
    int local_only;           // assignments outside the local window are dropped (not an error)
};

constexpr int kDispatchThreads = 1024;

inline size_t dispatch_smem(int E) { return sizeof(int) * ((size_t)2 * (E + 1) + (size_t)32 * E + 64); }

// Dispatch, one CTA of 1024 threads (counting sort: per-expert counts, scans,
// a stable scatter in rounds of 1024 assignments).
__global__ void __launch_bounds__(kDispatchThreads) dispatch_kernel(DispatchParams p) {
    extern __shared__ __align__(16) int dsm[];
    const int E = p.E;
    int n = p.T * p.k;
    if (p.ep_flags) {
        const uint32_t want = *p.ep_epoch + 1;
        bool ok = true;
        if ((int)threadIdx.x < p.ep_G) ok = ep_wait_flag(p.ep_flags + threadIdx.x, want);
        // a rank that never delivered: no routed assignments (error flagged)
        if (__syncthreads_or(!ok)) {
            if (threadIdx.x == 0) atomicOr(&p.sched->err, (int)ERR_TIMEOUT);
            n = 0;
        }
        if (threadIdx.x == 0) *p.ep_epoch = want;
    }
    int* cnt = dsm;                  // [E+1]
    int* base = cnt + (E + 1);       // [E+1]
    int* wc = base + (E + 1);        // [32][E]
    int* wsum = wc + 32 * E;         // [64] scan scratch
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int e = tid; e <= E; e += kDispatchThreads) cnt[e] = 0;
    __syncthreads();
    const int lo = p.local_only ? p.first_expert : 0, hi = p.local_only ? p.first_expert + p.n_local : E;
    for (int a = tid; a < n; a += kDispatchThreads) {
        int e = p.topk_idx[a];
        if (e >= lo && e < hi) atomicAdd(&cnt[e], 1);
        else if (e < 0 || e >= E) atomicOr(&p.sched->err, (int)ERR_BOUNDS);
    }
    __syncthreads();
    // exclusive scans of the counts and of the "active local expert" flags:
    // warp w < 16 scans experts [32w, 32w+32)
    int c = 0, flag = 0, incl_c = 0, incl_f = 0;
    const int e_me = tid;
    if (warp < 16) {
        if (e_me < E) {
            c = cnt[e_me];
            flag = (c > 0 && e_me >= p.first_expert && e_me < p.first_expert + p.n_local) ? 1 : 0;
        }
        incl_c = c;
        incl_f = flag;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            int a = __shfl_up_sync(0xffffffffu, incl_c, o), b = __shfl_up_sync(0xffffffffu, incl_f, o);
            if (lane >= o) { incl_c += a; incl_f += b; }
        }
        if (lane == 31) { wsum[warp] = incl_c; wsum[32 + warp] = incl_f; }
    }
    __syncthreads();
    if (warp == 0) {
        int a = lane < 16 ? wsum[lane] : 0, b = lane < 16 ? wsum[32 + lane] : 0;
        int ia = a, ib = b;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            int x = __shfl_up_sync(0xffffffffu, ia, o), y = __shfl_up_sync(0xffffffffu, ib, o);
            if (lane >= o) { ia += x; ib += y; }
        }
        if (lane < 16) { wsum[lane] = ia - a; wsum[32 + lane] = ib - b; }
        if (lane == 15) { wsum[48] = ia; wsum[49] = ib; }
    }
    __syncthreads();
    if (warp < 16 && e_me < E) {
        int ex = wsum[warp] + incl_c - c;
        base[e_me] = ex;
        p.offsets[e_me] = ex;
        if (flag) p.active[wsum[32 + warp] + incl_f - 1] = e_me;
    }
    if (tid == 0) {
        int total = wsum[48], na = wsum[49];
        p.offsets[E] = total;
        if (p.has_shared) p.active[na] = E;
        p.sched->n_active = na;
        for (int q = 0; q < 4; q++) p.sched->ctr[q] = 0;
    }
    __syncthreads();
    // stable scatter, 1024 assignments per round
    for (int r0 = 0; r0 < n; r0 += kDispatchThreads) {
        const int a = r0 + tid;
        int e = a < n ? p.topk_idx[a] : -1;
        if (e >= hi || e < lo) e = -1;
        const unsigned peers = __match_any_sync(0xffffffffu, e);
        const int rank_w = __popc(peers & ((1u << lane) - 1));
        const int leader = __ffs(peers) - 1;
        int* row = wc + warp * E;
        for (int i = lane; i < E; i += 32) row[i] = 0;
        __syncwarp();
        if (e >= 0 && lane == leader) row[e] = __popc(peers);
        __syncthreads();
        if (e >= 0) {
            int before = 0;
            for (int w = 0; w < warp; w++) before += wc[w * E + e];
            const int pos = base[e] + before + rank_w;
            p.perm[pos] = a;
            p.inv_perm[a] = pos;
            p.pos_tok[pos] = a / p.k;
        }
        __syncthreads();
        if (e >= 0 && lane == leader) atomicAdd(&base[e], __popc(peers));
        __syncthreads();
    }
    // per active slot: expert, first position, tokens, first token
    const int na = p.sched->n_active;
    for (int sl = tid; sl < na; sl += kDispatchThreads) {
        const int e = p.active[sl], off = p.offsets[e];
        p.slot_info[sl] = make_int4(e, off, p.offsets[e + 1] - off, p.perm[off] / p.k);
    }
    if (tid == 0 && p.has_shared) p.slot_info[na] = make_int4(E, 0, p.T_sh, 0);
}

// Top-k and dispatch of a batch of T <= 32 tokens (n = T*k <= 256
// assignments) in one CTA of 1024 threads: warp t ranks token t
// (topk_warp), then the dispatch is computed directly, one thread per
// assignment a (expert e_a): pos(a) = #{b : e_b < e_a} + #{b < a : e_b == e_a}
// (stable inside an expert), offsets[e] = #{b : e_b < e}; the active list
// holds the local experts with assignments, ascending.  The same positions,
// offsets and slots as dispatch_kernel, with rolled loops over 128-bit
// shared loads and three block barriers (the code runs cold once per forward).
constexpr int kFusedTopkMaxT = 32;

inline size_t topk_dispatch_smem(int E, int T) { return (size_t)2 * sizeof(float) * min(T, kFusedTopkMaxT) * E; }

template <int J>
__global__ void __launch_bounds__(kDispatchThreads) topk_dispatch_kernel(DispatchParams p, TopkParams tp) {
    extern __shared__ __align__(16) float tsm[];   // [T][2][E]: weight sources, keys
    __shared__ uint64_t tab[32];
    // assignment arrays padded to a multiple of 4 with INT_MAX (counts nowhere)
    __shared__ __align__(16) int asg[kFusedTopkMaxT * kMaxK];   // expert of assignment a
    __shared__ __align__(16) int act[kFusedTopkMaxT * kMaxK];   // expert of a first local assignment, else INT_MAX
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int E = p.E, k = tp.k, n = tp.T * k, n4 = (n + 3) / 4;
    if (tid < 32) tab[tid] = kExpfTabDev[tid];
    if (tid >= n && tid < 4 * n4) asg[tid] = act[tid] = 0x7fffffff;
    __syncthreads();
    if (warp < tp.T) {
        float* sv = tsm + (size_t)warp * 2 * E;
        const int e = topk_warp<J>(tp, warp, lane, sv, reinterpret_cast<uint32_t*>(sv + E), tab);
        if (lane < k) asg[warp * k + lane] = e;
    }
    __syncthreads();
    const int4* a4 = reinterpret_cast<const int4*>(asg);
    const int lo = p.local_only ? p.first_expert : 0, hi = p.local_only ? p.first_expert + p.n_local : E;
#pragma unroll 1
    for (int e = tid; e <= E; e += kDispatchThreads) {
        int c = 0;
#pragma unroll 2
        for (int b = 0; b < n4; b++) {
            const int4 q = a4[b];
            c += (q.x >= lo && q.x < hi && q.x < e) + (q.y >= lo && q.y < hi && q.y < e) +
                 (q.z >= lo && q.z < hi && q.z < e) + (q.w >= lo && q.w < hi && q.w < e);
        }
        p.offsets[e] = c;
    }
    int e = -1, below = 0, rank = 0, cnt = 0;
    if (tid < n) {
        e = asg[tid];
        if (e < 0 || e >= E) atomicOr(&p.sched->err, (int)ERR_BOUNDS);
        if (e < lo || e >= hi) e = -1;
        if (e >= 0) {
#pragma unroll 2
            for (int b = 0; b < n4; b++) {
                const int4 q = a4[b];
                below += (q.x >= lo && q.x < e) + (q.y >= lo && q.y < e) + (q.z >= lo && q.z < e) + (q.w >= lo && q.w < e);
                cnt += (q.x == e) + (q.y == e) + (q.z == e) + (q.w == e);
                const int b0 = 4 * b;
                rank += (b0 < tid && q.x == e) + (b0 + 1 < tid && q.y == e) + (b0 + 2 < tid && q.z == e) +
                        (b0 + 3 < tid && q.w == e);
            }
        }
    }
    const bool is_act = e >= 0 && rank == 0 && e >= p.first_expert && e < p.first_expert + p.n_local;
    if (tid < n) act[tid] = is_act ? e : 0x7fffffff;
    const int nd = __syncthreads_count(is_act);
    if (e >= 0) {
        const int pos = below + rank;
        p.perm[pos] = tid;
        p.inv_perm[tid] = pos;
        p.pos_tok[pos] = tid / k;
        if (is_act) {
            const int4* c4 = reinterpret_cast<const int4*>(act);
            int dbelow = 0;
#pragma unroll 2
            for (int b = 0; b < n4; b++) {
                const int4 q = c4[b];
                dbelow += (q.x < e) + (q.y < e) + (q.z < e) + (q.w < e);
            }
            p.active[dbelow] = e;
            p.slot_info[dbelow] = make_int4(e, below, cnt, tid / k);
        }
    }
    if (tid == 0) {
        if (p.has_shared) {
            p.active[nd] = E;
            p.slot_info[nd] = make_int4(E, 0, p.T_sh, 0);
        }
        p.sched->n_active = nd;
        for (int q = 0; q < 4; q++) p.sched->ctr[q] = 0;
    }
}

// ---------------------------------------------------------------------------
// Lane-major router rows for the fused router: row e is stored as 8 lanes of P
// floats, lane j holding columns j, j+8, j+16, ... (the columns of one
// Vector256 lane of SimdMath.DotF32) contiguously, zero-padded to P >= d/8
// with P = 4 mod 32 (16-byte aligned, 8 lanes on distinct banks).
__host__ __device__ inline int route_lane_pitch(int d) { return (d / 8 + 27) / 32 * 32 + 4; }

__global__ void router_lane_major_kernel(const float* __restrict__ w, float* __restrict__ wp, int E, int d) {
    const int P = route_lane_pitch(d), m8 = d / 8;
    const long long total = (long long)E * 8 * P;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
        const int e = (int)(i / (8 * P));
        const int r = (int)(i - (long long)e * 8 * P), j = r / P, m = r - j * P;
        wp[i] = m < m8 ? w[(size_t)e * d + 8 * m + j] : 0.f;
    }
}

// acc + sum over m < nm of a[m]*b[m], in that order, from lane-major rows
// (16-byte aligned, nm % 4 == 0): one 128-bit load covers four steps, and the
// loads of the next 16 steps are in flight while the current adds run.
__device__ __forceinline__ float lane_chain4(const float* __restrict__ a, const float* __restrict__ b, int nm,
                                             float acc) {
    const float4* a4 = reinterpret_cast<const float4*>(a);
    const float4* b4 = reinterpret_cast<const float4*>(b);
    const int n4 = nm / 4;
    int q = 0;
    if (n4 >= 8) {
        float4 A[4], B[4];
#pragma unroll
        for (int u = 0; u < 4; u++) { A[u] = a4[u]; B[u] = b4[u]; }
        for (q = 4; q + 4 <= n4; q += 4) {
            float4 An[4], Bn[4];
#pragma unroll
            for (int u = 0; u < 4; u++) { An[u] = a4[q + u]; Bn[u] = b4[q + u]; }
#pragma unroll
            for (int u = 0; u < 4; u++) {
                acc = __fadd_rn(acc, __fmul_rn(A[u].x, B[u].x));
                acc = __fadd_rn(acc, __fmul_rn(A[u].y, B[u].y));
                acc = __fadd_rn(acc, __fmul_rn(A[u].z, B[u].z));
                acc = __fadd_rn(acc, __fmul_rn(A[u].w, B[u].w));
                A[u] = An[u];
                B[u] = Bn[u];
            }
        }
#pragma unroll
        for (int u = 0; u < 4; u++) {
            acc = __fadd_rn(acc, __fmul_rn(A[u].x, B[u].x));
            acc = __fadd_rn(acc, __fmul_rn(A[u].y, B[u].y));
            acc = __fadd_rn(acc, __fmul_rn(A[u].z, B[u].z));
            acc = __fadd_rn(acc, __fmul_rn(A[u].w, B[u].w));
        }
    }
    for (; q < n4; q++) {
        const float4 x = a4[q], y = b4[q];
        acc = __fadd_rn(acc, __fmul_rn(x.x, y.x));
        acc = __fadd_rn(acc, __fmul_rn(x.y, y.y));
        acc = __fadd_rn(acc, __fmul_rn(x.z, y.z));
        acc = __fadd_rn(acc, __fmul_rn(x.w, y.w));
    }
    return acc;
}

// ---------------------------------------------------------------------------
// Router logits for batches beyond the single-launch routers, tiled.  A CTA
// owns NTG*TT tokens x NEG*TE experts with NTG*NEG*8 threads; thread (token
// group tg, expert group eg, lane j) runs the TT*TE chains of lane j for its
// tokens x experts (SimdMath.DotF32's lane j: acc + w*x over columns j, j+8,
// ... in order, products and sums rounded separately), so the logits stay
// bit-exact.  Chunks of KC steps (8*KC columns) of the token rows
// (row-major) and of the experts' lane-major router rows (router_lm) stream
// into NS shared buffers with cp.async, NS-1 chunks in flight (the router
// rows come from DRAM after the caches turned over, and a chain consumes a
// chunk in a fraction of that latency); a 128-bit load covers four steps of
// one expert, the token columns of lane j are four conflict-free scalar
// loads (a warp holds one token group, so its expert groups read the same
// token words).  The host picks the largest tile whose grid still covers the
// SMs: the T*E*8 chains of d/8 dependent adds cannot be split, so at small T
// the chains must spread over CTAs, and at large T more chains per thread
// keep the FP32 pipes busy with fewer shared loads per product.
template <int TT, int TE, int NTG, int NEG, int KC, int NS>
struct LMTile {
    static constexpr int kThreads = NTG * NEG * 8, kT = NTG * TT, kE = NEG * TE;
    static constexpr int kXPitch = 8 * KC + 4;   // floats per token row of a chunk (4 banks apart)
    static constexpr int kWPitch = KC + 4;       // floats per (expert, lane): the 8 lanes start 4 banks apart
    static constexpr int kBuf = kT * kXPitch + kE * 8 * kWPitch;   // floats of one chunk buffer
    static constexpr size_t smem() { return sizeof(float) * NS * kBuf; }
    static_assert(NEG % 4 == 0, "a warp spans one token group");
    static_assert(KC % 4 == 0 && (KC & (KC - 1)) == 0, "chunks of a power-of-two number of 4-step groups");
    static_assert(NS >= 2 && kT * kE * 8 <= NS * kBuf, "lane sums fit the chunk buffers");
};

template <int TT, int TE, int NTG, int NEG, int KC, int NS>
__global__ void __launch_bounds__(NTG * NEG * 8, 1024 / (NTG * NEG * 8))
logits_lm_kernel(const float* __restrict__ xn, const float* __restrict__ router_lm, const float* __restrict__ offset,
                 float* __restrict__ logits, int T, int d, int E) {
    using Tl = LMTile<TT, TE, NTG, NEG, KC, NS>;
    constexpr int NT = Tl::kThreads, KT = Tl::kT, KE = Tl::kE, XPt = Tl::kXPitch, WPt = Tl::kWPitch;
    constexpr int XQ = 2 * KC, WQ = KC / 4;     // 16-byte pieces per token row / per (expert, lane) row
    constexpr int XP = KT * XQ, WP = KE * 8 * WQ;
    extern __shared__ __align__(16) float lsm[];
    const int tid = threadIdx.x, j = tid & 7, eg = (tid >> 3) % NEG, tg = tid / (8 * NEG);
    const int t0 = blockIdx.x * KT, e0 = blockIdx.y * KE;
    const int nm = d / 8, P = route_lane_pitch(d);            // d % 32 == 0: nm % 4 == 0
    const int nch = (nm + KC - 1) / KC;
    auto load = [&](int c) {
        if (c < nch) {
            float* X = lsm + (c % NS) * Tl::kBuf;
            float* W = X + KT * XPt;
#pragma unroll
            for (int u = 0; u < (XP + NT - 1) / NT; u++) {
                const int i = tid + u * NT, r = i / XQ, q = i % XQ;     // token row r, piece q
                if (XP % NT == 0 || i < XP) {
                    const int col = 8 * KC * c + 4 * q;
                    float* dst = X + r * XPt + 4 * q;
                    if (t0 + r < T && col < d) cp_async16(dst, xn + (size_t)(t0 + r) * d + col);
                    else *reinterpret_cast<float4*>(dst) = make_float4(0.f, 0.f, 0.f, 0.f);
                }
            }
#pragma unroll
            for (int u = 0; u < (WP + NT - 1) / NT; u++) {
                const int i = tid + u * NT, row = i / WQ, q = i % WQ;    // row = expert * 8 + lane
                if (WP % NT == 0 || i < WP) {
                    const int e = e0 + (row >> 3), m = KC * c + 4 * q;
                    float* dst = W + row * WPt + 4 * q;
                    if (e < E && m < nm) cp_async16(dst, router_lm + ((size_t)e * 8 + (row & 7)) * P + m);
                    else *reinterpret_cast<float4*>(dst) = make_float4(0.f, 0.f, 0.f, 0.f);
                }
            }
        }
        cp_async_commit();   // empty groups past the end keep the accounting uniform
    };
    float acc[TT][TE];
#pragma unroll
    for (int a = 0; a < TT; a++)
#pragma unroll
        for (int b = 0; b < TE; b++) acc[a][b] = 0.f;
#pragma unroll
    for (int c = 0; c < NS - 1; c++) load(c);
    for (int c = 0; c < nch; c++) {
        load(c + NS - 1);
        cp_async_wait<NS - 1>();   // chunk c has landed
        __syncthreads();
        const float* X = lsm + (c % NS) * Tl::kBuf;
        const float* W = X + KT * XPt;
        const int steps = min(KC, nm - KC * c);   // a multiple of 4
        for (int q = 0; q < steps / 4; q++) {
            float x[TT][4];
#pragma unroll
            for (int a = 0; a < TT; a++)
#pragma unroll
                for (int s = 0; s < 4; s++) x[a][s] = X[(TT * tg + a) * XPt + 8 * (4 * q + s) + j];
#pragma unroll
            for (int b = 0; b < TE; b++) {
                const float4 w = *reinterpret_cast<const float4*>(W + ((TE * eg + b) * 8 + j) * WPt + 4 * q);
#pragma unroll
                for (int a = 0; a < TT; a++) {
                    acc[a][b] = __fadd_rn(acc[a][b], __fmul_rn(w.x, x[a][0]));
                    acc[a][b] = __fadd_rn(acc[a][b], __fmul_rn(w.y, x[a][1]));
                    acc[a][b] = __fadd_rn(acc[a][b], __fmul_rn(w.z, x[a][2]));
                    acc[a][b] = __fadd_rn(acc[a][b], __fmul_rn(w.w, x[a][3]));
                }
            }
        }
        __syncthreads();   // buffer c % NS is refilled by the next iteration
    }
    cp_async_wait<0>();
    // lane sums in order: red[token][expert][lane]
    float* red = lsm;
#pragma unroll
    for (int a = 0; a < TT; a++)
#pragma unroll
        for (int b = 0; b < TE; b++) red[((TT * tg + a) * KE + TE * eg + b) * 8 + j] = acc[a][b];
    __syncthreads();
    for (int i = tid; i < KT * KE; i += NT) {
        const int tt = i / KE, ee = i - tt * KE, t = t0 + tt, e = e0 + ee;
        if (t < T && e < E) {
            float s = hsum8_seq(red + (size_t)i * 8);
            if (offset) s = __fadd_rn(s, offset[e]);
            logits[(size_t)t * E + e] = s;
        }
    }
}

// The tiles the host chooses from, largest first (TT, TE, NTG, NEG, KC, NS):
// 32 x 32 (16 chains per thread, two CTAs per SM), 16 x 16 (16), 8 x 8 (4),
// 4 x 8 (2); the smaller tiles take longer chunks and deeper pipelines.
#define QRM_LM_TILES(X) X(4, 4, 8, 8, 16, 2) X(4, 4, 4, 4, 16, 5) X(2, 2, 4, 4, 32, 6) X(1, 2, 4, 4, 32, 6)

// ---------------------------------------------------------------------------
// Fused small-T router: RMSNorm, router logits, top-k and dispatch in one
// launch.  CTA b owns experts [kRouteEPC*b, +kRouteEPC).  Thread 0 bulk-copies
// the token rows, the norm weights and the CTA's router rows into shared
// memory (one copy per row, each group on its own mbarrier, so the RMSNorm
// chains start as soon as the token rows land); every CTA recomputes the
// RMSNorm of its T tokens and writes its slice of the xn columns.  The last
// CTA to finish its logits (arrival counter in the schedule) ranks every
// token's logits and dispatches, so routing costs one launch.
// Shared memory: W[EPC][d + 4] | X[T][d] | NW[d] | red | scl | barriers; the
// top-k / dispatch scratch of the last CTA reuses W.
constexpr int kRouteFusedMaxT = 4;   // one warp per token in the tail; T*k <= 32

__host__ __device__ inline size_t route_fused_main_floats(int d, int T, int E) {
    // W[EPC][8P] | X[T][d] | XP[T][8P] | NW | red | scl (padded to 4) | bias[E] (padded to 4) | exp table
    const size_t P8 = (size_t)8 * route_lane_pitch(d);
    return (size_t)kRouteEPC * P8 + (size_t)T * d + (size_t)T * P8 + d + (size_t)T * kRouteEPC * 8 +
           (size_t)(T + 3) / 4 * 4 + (size_t)(E + 3) / 4 * 4 + 64;
}
inline size_t route_tail_smem(int E, int T) {
    // sv, key [T][E] | asg [32] | rsel [kRouteFusedMaxT][kMaxK] | wred [T][4]
    return sizeof(float) * (size_t)2 * T * E + sizeof(int) * (32 + 4 * 8 + 16);
}
inline size_t route_fused_smem(int d, int T, int E) {
    return (sizeof(float) * route_fused_main_floats(d, T, E) + 15) / 16 * 16 + 4 * 8;   // + 3 mbarriers
}
inline int route_fused_max_tokens(int d, int E) {
    int t = kRouteFusedMaxT;
    while (t > 0 && (route_fused_smem(d, t, E) > 220 * 1024 ||
                     route_tail_smem(E, t) > sizeof(float) * (size_t)kRouteEPC * 8 * route_lane_pitch(d)))
        t--;
    return E <= kMaxE ? t : 0;
}

struct RouteFusedParams {
    RouteParams r;             // r.router unused: rows come from router_lm
    const float* router_lm;    // [E][8][P] lane-major router rows
    TopkParams tp;
    DispatchParams dp;
};


// Top-k of every token and the dispatch of the n = T*k <= 32 assignments.
// Scores: the whole CTA (softmax: StreamingEngine.cs:642-647 with the
// sequential sum; GLM sigmoid + bias: 730-767).  Selection: one warp per token,
// k rounds of "largest key, lowest index" over registers.  Dispatch, computed
// directly: offsets[e] = #assignments with expert < e, pos(a) = offsets[e_a] +
// #{b < a : e_b == e_a} (stable), active = local experts with assignments,
// ascending.
// scratch: sv / key / asg / wred (may alias consumed data); bias: E floats of
// tp.bias staged in shared memory (or null); tab: the exp table in shared memory
template <int J>
__device__ void route_tail(const TopkParams& tp, const DispatchParams& p, uint8_t* scratch, const float* bias,
                           const uint64_t* tab) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int NW = kRouteThreads / 32;
    const int E = p.E, T = tp.T, k = tp.k, n = T * k;
    float* sv = reinterpret_cast<float*>(scratch);                       // [T][E] weight sources
    uint32_t* key = reinterpret_cast<uint32_t*>(sv + (size_t)T * E);     // [T][E] ranking keys
    int* asg = reinterpret_cast<int*>(key + (size_t)T * E);              // [32] expert of assignment a
    float* wred = reinterpret_cast<float*>(asg + 32 + kRouteFusedMaxT * kMaxK);   // [T][NW] max / sum scratch
    if (!tp.sigmoid) {
        // max from float.MinValue (comparisons skip NaN like the reference loop)
        for (int t = 0; t < T; t++) {
            float mx = -3.40282347e+38f;
            for (int i = tid; i < E; i += kRouteThreads) {
                const float a = __ldcg(tp.logits + (size_t)t * E + i);
                sv[t * E + i] = a;
                if (a > mx) mx = a;
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) { const float b = __shfl_xor_sync(0xffffffffu, mx, o); if (b > mx) mx = b; }
            if (lane == 0) wred[t * NW + warp] = mx;
        }
        __syncthreads();
        for (int t = 0; t < T; t++) {
            float mx = wred[t * NW];
#pragma unroll
            for (int w = 1; w < NW; w++) if (wred[t * NW + w] > mx) mx = wred[t * NW + w];
            for (int i = tid; i < E; i += kRouteThreads) sv[t * E + i] = expf_glibc_t(__fsub_rn(sv[t * E + i], mx), tab);
        }
        __syncthreads();
        if (tid < T) {   // sequential sum in index order
            const float* e = sv + tid * E;
            float sum = 0.f;
            int i = 0;
            for (; i + 16 <= E; i += 16) {
                float q[16];
#pragma unroll
                for (int u = 0; u < 16; u++) q[u] = e[i + u];
#pragma unroll
                for (int u = 0; u < 16; u++) sum = __fadd_rn(sum, q[u]);
            }
            for (; i < E; i++) sum = __fadd_rn(sum, e[i]);
            wred[tid * NW] = __fdiv_rn(1.f, sum);
        }
        __syncthreads();
        for (int i = tid; i < T * E; i += kRouteThreads) {
            const float q = __fmul_rn(sv[i], wred[(i / E) * NW]);
            sv[i] = q;
            key[i] = rank_key(q);
        }
    } else {
        for (int i = tid; i < T * E; i += kRouteThreads) {
            const int e = i - (i / E) * E;
            const float sg = __fdiv_rn(1.f, __fadd_rn(1.f, expf_glibc_t(-__ldcg(tp.logits + i), tab)));
            sv[i] = sg;
            key[i] = rank_key(bias ? __fadd_rn(sg, bias[e]) : sg);
        }
    }
    __syncthreads();
    // selection, one warp per token: lane l holds the keys of candidates
    // l, l+32, ... in registers; k rounds of "largest key, then lowest index"
    // (value descending, index ascending: a total order) by two warp
    // reductions each, with no block-wide synchronisation
    int* rsel = asg + 32;   // [T][kMaxK] (the weight scratch follows)
    if (warp < T) {
        const int t = warp;
        const uint32_t* kt = key + (size_t)t * E;
        uint32_t kc[J];   // key + 1 of candidate lane + 32 i (0: none or taken)
#pragma unroll
        for (int i = 0; i < J; i++) {
            const int c = lane + 32 * i;
            kc[i] = c < E ? kt[c] + 1u : 0u;   // keys are below 0xFF800001: no wrap
        }
        const int e = warp_select<J>(kc, k, lane);
        if (lane < k) rsel[t * kMaxK + lane] = e;
    }
    __syncthreads();
    if (warp < T) {
        // weights of token t = warp: the sum in rank order on lane 0 (bit-exact
        // sequence), then one lane per selected expert
        const int t = warp;
        const int e = lane < k ? rsel[t * kMaxK + lane] : 0;
        const float se = lane < k ? sv[t * E + e] : 0.f;
        float sum = 0.f;
#pragma unroll 1
        for (int r = 0; r < k; r++) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, se, r));
        if (lane < k) {
            float wv;
            if (!tp.sigmoid) {
                wv = __fdiv_rn(se, sum <= 0.f ? 1.f : sum);
            } else {
                const float inv2 = __fdiv_rn(1.f, __fadd_rn(sum, 1e-20f));
                wv = __fmul_rn(__fmul_rn(se, inv2), tp.routed_scale);
            }
            tp.topk_idx[(size_t)t * k + lane] = e;
            tp.topk_w[(size_t)t * k + lane] = wv;
            asg[t * k + lane] = e;
        }
    }
    for (int a = n + tid; a < 32; a += kRouteThreads) asg[a] = 0x7fffffff;   // padding sorts last
    __syncthreads();
    // Compact loops from here on (not unrolled): this code runs on one CTA
    // once per forward, usually with its instructions cold in every cache, so
    // its length costs more than its instruction count.
#pragma unroll 1
    for (int e = tid; e <= E; e += kRouteThreads) {
        int c = 0;
#pragma unroll 1
        for (int a = 0; a < n; a++) c += asg[a] < e ? 1 : 0;
        p.offsets[e] = c;
    }
    if (warp == 0) {
        const int a = lane;
        const int e = asg[lane];   // 0x7fffffff past n
        const unsigned peers = __match_any_sync(0xffffffffu, e);
        const bool first = a < n && lane == __ffs(peers) - 1;
        const bool local = a < n && e >= p.first_expert && e < p.first_expert + p.n_local;
        const unsigned firsts = __ballot_sync(0xffffffffu, first && local);
        int below = 0, dbelow = 0;
#pragma unroll 1
        for (int b = 0; b < n; b++) {
            const int eb = asg[b];
            below += eb < e ? 1 : 0;
            dbelow += ((firsts >> b) & 1u) && eb < e ? 1 : 0;
        }
        if (a < n) {
            const int pos = below + __popc(peers & ((1u << lane) - 1));   // stable inside an expert
            p.perm[pos] = a;
            p.inv_perm[a] = pos;
            p.pos_tok[pos] = a / p.k;
            if (first && local) {
                p.active[dbelow] = e;
                p.slot_info[dbelow] = make_int4(e, below, __popc(peers), a / p.k);
            }
        }
        if (lane == 0) {
            const int nd = __popc(firsts);
            if (p.has_shared) {
                p.active[nd] = E;
                p.slot_info[nd] = make_int4(E, 0, p.T_sh, 0);
            }
            p.sched->n_active = nd;
            for (int q = 0; q < 4; q++) p.sched->ctr[q] = 0;
        }
    }
}

__global__ void __launch_bounds__(kRouteThreads, 1)
route_fused_kernel(RouteFusedParams fp) {
    extern __shared__ __align__(16) float smem[];
    const RouteParams& p = fp.r;
    const int d = p.d, T = p.T;
    const int P = route_lane_pitch(d), P8 = 8 * P, m8 = d / 8;   // d % 32 == 0 (host check)
    const int e0 = blockIdx.x * kRouteEPC;
    const int ne = min(kRouteEPC, p.E - e0);
    float* W = smem;                        // [EPC][8][P] lane-major router rows
    float* X = W + kRouteEPC * P8;          // [T][d] token rows as given
    float* XP = X + T * d;                  // [T][8][P] normalised rows, lane-major
    float* NW = XP + T * P8;                // [d]
    float* red = NW + d;                    // [T*EPC*8]
    float* scl = red + T * kRouteEPC * 8;   // [T]
    float* sbias = scl + (T + 3) / 4 * 4;   // [E] (GLM router bias, for the last CTA)
    uint64_t* stab = reinterpret_cast<uint64_t*>(sbias + (p.E + 3) / 4 * 4);   // [32] exp table
    uint64_t* bar = reinterpret_cast<uint64_t*>(
        reinterpret_cast<uint8_t*>(smem) + (sizeof(float) * route_fused_main_floats(d, T, p.E) + 15) / 16 * 16);
    __shared__ int s_flag;                  // bit 0: a wait gave up; bit 1: last CTA
    const int tid = threadIdx.x;
    const int d8 = d / 8 * 8;
    const bool norm = p.apply_norm != 0;
    const bool has_nw = norm && p.norm_w != nullptr;

    pdl_trigger();   // the expert kernel may be scheduled; it waits for this grid
    if (tid == 0) {
        s_flag = 0;
        for (int i = 0; i < 3; i++) mbar_init(&bar[i], 1);
        fence_barrier_init();
        // token rows, then norm weights, then router rows (16-byte aligned rows)
        const uint32_t rb = (uint32_t)(sizeof(float) * d);
        mbar_arrive_expect_tx(&bar[0], rb * T);
        for (int t = 0; t < T; t++) bulk_g2s(X + t * d, p.x + (size_t)t * d, rb, &bar[0]);
        if (has_nw) {
            mbar_arrive_expect_tx(&bar[1], rb);
            bulk_g2s(NW, p.norm_w, rb, &bar[1]);
        } else {
            mbar_arrive(&bar[1]);
        }
        const uint32_t wb = (uint32_t)(sizeof(float) * P8);
        mbar_arrive_expect_tx(&bar[2], wb * ne);
        for (int e = 0; e < ne; e++) bulk_g2s(W + e * P8, fp.router_lm + (size_t)(e0 + e) * P8, wb, &bar[2]);
    }
    // what the last CTA's ranking needs, staged while the chains run
    if (fp.tp.bias) {
        for (int i = 4 * tid; i + 4 <= p.E; i += 4 * kRouteThreads) cp_async16(sbias + i, fp.tp.bias + i);
        if (tid < (p.E & 3)) sbias[(p.E & ~3) + tid] = fp.tp.bias[(p.E & ~3) + tid];
    }
    cp_async_commit();
    const uint64_t tabv = kExpfTabDev[tid & 31];   // stored after the chains (hides the load)
    __syncthreads();
    // bounded wait on group g by every thread; a timeout is reported through
    // the schedule's error flags (qrm_sync returns QRM_E_TIMEOUT)
    auto wait_group = [&](int g) {
        if (!mbar_wait(&bar[g], 0u)) atomicOr(&s_flag, 1);
    };

    // RMSNorm chains, thread (t, j) for t < T, j < 8
    wait_group(0);
    // chain group g (token or (token, expert)) -> warp g % 4, lanes 8*(g/4)..+7,
    // so the groups issue from different schedulers
    const int cg = (tid >> 5) + 4 * ((tid & 31) >> 3), cj = tid & 7;
    if (norm && cg < T) red[cg * 8 + cj] = lane_chain_sq(X + cg * d, cj, d8, 0.f);
    __syncthreads();
    if (norm) {
        if (tid < T) {
            const float* xr = X + tid * d;
            float ss = 0.f;
            int i = 0;
            if (d >= 8) { ss = hsum8_seq(red + tid * 8); i = d8; }
            for (; i < d; i++) ss = __fadd_rn(ss, __fmul_rn(xr[i], xr[i]));
            const float v = __fadd_rn(__fdiv_rn(ss, (float)d), p.eps);
            scl[tid] = __fdiv_rn(1.f, __fsqrt_rn(v));
        }
        wait_group(1);
    } else {
        wait_group(1);
    }
    __syncthreads();
    // normalise into the lane-major XP and write this CTA's slice of xn
    {
        const int d4 = d / 4;
        const int c0 = (int)((long long)d4 * blockIdx.x / gridDim.x), c1 = (int)((long long)d4 * (blockIdx.x + 1) / gridDim.x);
        const float4* nw4 = reinterpret_cast<const float4*>(NW);
        for (int t = 0; t < T; t++) {
            const float sc = norm ? scl[t] : 1.f;
            const float4* xr = reinterpret_cast<const float4*>(X + t * d);
            float* xp = XP + t * P8;
            for (int c = tid; c < d4; c += kRouteThreads) {
                float4 v = xr[c];
                if (norm) {
                    v.x = __fmul_rn(v.x, sc); v.y = __fmul_rn(v.y, sc); v.z = __fmul_rn(v.z, sc); v.w = __fmul_rn(v.w, sc);
                    if (has_nw) {
                        const float4 w = nw4[c];
                        v.x = __fmul_rn(v.x, w.x); v.y = __fmul_rn(v.y, w.y); v.z = __fmul_rn(v.z, w.z); v.w = __fmul_rn(v.w, w.w);
                    }
                }
                // columns 4c..4c+3 -> lanes (4c & 7) + i, position (4c) >> 3
                const int j0 = (4 * c) & 7, m = (4 * c) >> 3;
                xp[(j0 + 0) * P + m] = v.x;
                xp[(j0 + 1) * P + m] = v.y;
                xp[(j0 + 2) * P + m] = v.z;
                xp[(j0 + 3) * P + m] = v.w;
                if (c >= c0 && c < c1) reinterpret_cast<float4*>(p.xn + (size_t)t * d)[c] = v;
            }
        }
    }
    wait_group(2);
    __syncthreads();
    // logit chains: thread (t, e, j)
    {
        const int lt = cg / kRouteEPC, le = cg - lt * kRouteEPC;
        if (lt < T && le < ne) red[cg * 8 + cj] = lane_chain4(W + le * P8 + cj * P, XP + lt * P8 + cj * P, m8, 0.f);
    }
    __syncthreads();
    if (tid < T * ne) {
        const int t = tid / ne, e = tid - t * ne;
        float s = hsum8_seq(red + (t * kRouteEPC + e) * 8);   // no tail columns: d % 8 == 0
        if (p.offset) s = __fadd_rn(s, p.offset[e0 + e]);
        p.logits[(size_t)t * p.E + e0 + e] = s;
        __threadfence();
    }
    // the last CTA to arrive ranks and dispatches
    if (tid < 32) stab[tid] = tabv;
    __syncthreads();
    if (tid == 0) {
        if (s_flag & 1) atomicOr(&fp.dp.sched->err, (int)ERR_TIMEOUT);
        __threadfence();
        if (atomicAdd(&fp.dp.sched->route_arrivals, 1) == (int)gridDim.x - 1) s_flag |= 2;
    }
    __syncthreads();
    if (!(s_flag & 2)) return;
    __threadfence();
    cp_async_wait<0>();
    __syncthreads();
    const float* bias = fp.tp.bias ? sbias : nullptr;
    if (p.E <= 256) route_tail<8>(fp.tp, fp.dp, reinterpret_cast<uint8_t*>(smem), bias, stab);
    else route_tail<kMaxE / 32>(fp.tp, fp.dp, reinterpret_cast<uint8_t*>(smem), bias, stab);
    if (tid == 0) fp.dp.sched->route_arrivals = 0;
}

}  // namespace qrm
