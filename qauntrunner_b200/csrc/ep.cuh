// ep.cuh -- expert-parallel data movement around the NCCL exchanges.
//
// G ranks, one process per GPU, each holding the routed experts
// [rank*E/G, (rank+1)*E/G) and a replica of norm, router and shared expert.
// Per forward every rank routes its own T tokens, all-gathers (normalised
// token, top-k indices, top-k weights) records, runs its experts for the
// G*T gathered tokens, returns each expert output row to the owner of its
// token, and the owner adds the rows in slot order.  The kernels here pack and
// unpack those messages; the exchanges are ncclAllGather and grouped
// ncclSend / ncclRecv in qrmoe.cu.
//
// Message layouts (f32 words):
//   record of token t: xn[d] | top-k indices[k] (int32 bits) | top-k weights[k]
//   output block for owner q: [T*k][d] rows, row t*k+j = expert output of q's
//   token t, slot j (only the rows whose expert this rank holds are written;
//   the owner reads exactly those).
#pragma once
#include "common.cuh"

namespace qrm {

__global__ void ep_pack_records_kernel(const float* __restrict__ xn, const int32_t* __restrict__ idx,
                                       const float* __restrict__ w, int T, int d, int k, float* __restrict__ rec) {
    const int W = d + 2 * k;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < (long long)T * W;
         i += (long long)gridDim.x * blockDim.x) {
        const int t = (int)(i / W), c = (int)(i - (long long)t * W);
        float v;
        if (c < d) v = xn[(size_t)t * d + c];
        else if (c < d + k) v = __int_as_float(idx[t * k + (c - d)]);
        else v = w[t * k + (c - d - k)];
        rec[i] = v;
    }
}

__global__ void ep_unpack_records_kernel(const float* __restrict__ rec, int Tall, int d, int k,
                                         float* __restrict__ xn_all, int32_t* __restrict__ idx_all) {
    const int W = d + 2 * k;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < (long long)Tall * (d + k);
         i += (long long)gridDim.x * blockDim.x) {
        const int t = (int)(i / (d + k)), c = (int)(i - (long long)t * (d + k));
        const float v = rec[(size_t)t * W + c];
        if (c < d) xn_all[(size_t)t * d + c] = v;
        else idx_all[t * k + (c - d)] = __float_as_int(v);
    }
}

// Output rows of the local experts into the per-owner blocks: gathered
// assignment a = (owner q, local assignment i) -> block q, row i.
__global__ void ep_pack_outputs_kernel(const float* __restrict__ y, const int32_t* __restrict__ inv_perm,
                                       const int32_t* __restrict__ idx_all, int G, int T, int k, int d,
                                       int first, int n_local, float* __restrict__ send) {
    const int d4 = d / 4;
    const long long total = (long long)G * T * k * d4;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const long long a = i / d4;
        const int c = (int)(i - a * d4);
        const int e = idx_all[a];
        if (e < first || e >= first + n_local) continue;
        const int pos = inv_perm[a];
        reinterpret_cast<float4*>(send)[a * d4 + c] = reinterpret_cast<const float4*>(y)[(size_t)pos * d4 + c];
    }
}

// The owner's combine, in the reference's order: out = (x) + w_0 y_0 + ... +
// w_{k-1} y_{k-1} (+ shared), each product and sum rounded separately
// (combine_kernel's arithmetic); y_j comes from the block of the rank that
// holds expert idx[t][j] (experts per rank: epr).
__global__ void ep_combine_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                  const int32_t* __restrict__ idx, const float* __restrict__ recv,
                                  const float* __restrict__ ys, int T, int k, int d, int epr, float* __restrict__ out) {
    const int d4 = d / 4;
    const long long total = (long long)T * d4;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int t = (int)(i / d4), c = (int)(i - (long long)t * d4);
        float4 acc = x ? reinterpret_cast<const float4*>(x + (size_t)t * d)[c] : make_float4(0.f, 0.f, 0.f, 0.f);
        for (int j = 0; j < k; j++) {
            const float wj = w[t * k + j];
            const int q = idx[t * k + j] / epr;
            const float4 v = reinterpret_cast<const float4*>(recv + (((size_t)q * T + t) * k + j) * d)[c];
            acc.x = __fadd_rn(acc.x, __fmul_rn(wj, v.x));
            acc.y = __fadd_rn(acc.y, __fmul_rn(wj, v.y));
            acc.z = __fadd_rn(acc.z, __fmul_rn(wj, v.z));
            acc.w = __fadd_rn(acc.w, __fmul_rn(wj, v.w));
        }
        if (ys) {
            const float4 v = reinterpret_cast<const float4*>(ys + (size_t)t * d)[c];
            acc.x = __fadd_rn(acc.x, v.x);
            acc.y = __fadd_rn(acc.y, v.y);
            acc.z = __fadd_rn(acc.z, v.z);
            acc.w = __fadd_rn(acc.w, v.w);
        }
        reinterpret_cast<float4*>(out + (size_t)t * d)[c] = acc;
    }
}

}  // namespace qrm
