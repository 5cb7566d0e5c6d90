// combine.cuh -- weighted combine of the expert outputs, in slot order.
//
// Reference: SimdMath.AxpyF32 (SimdMath.cs:55-71), out = out + w*y, one call
// per selected expert in sorted order (StreamingEngine.cs:665, 710, 775),
// then the GLM shared expert with weight 1 (StreamingEngine.cs:788).  MoeFfn
// accumulates into the residual x; LegacyMoeInto / GlmMoeFfn start from 0.
// Each output element is written by one thread that adds the k products in
// slot order with separately rounded multiply and add, so the combine is
// deterministic and mirrors the reference's operation order (no atomics).
#pragma once
#include "common.cuh"

namespace qrm {

struct CombineParams {
    const float* x;          // residual [T x d] (ADD_RESIDUAL) or null
    const float* y;          // routed outputs, perm order [T*k x d]
    const float* ys;         // shared outputs [T x d] or null
    const int32_t* inv_perm; // [T*k]
    const float* topk_w;     // [T x k]
    float* out;              // [T x d]
    int T, k, d;
    // optional (qrm_forward's mapped host staging): block 0 also copies the
    // top-k and the error flags there once the predecessors are done
    const int32_t* topk_idx;  // [T x k]
    const int32_t* err;
    int32_t* copy_idx;
    float* copy_w;
    int32_t* copy_err;
};

__global__ void combine_kernel(CombineParams p) {
    pdl_wait();   // the expert outputs of the predecessor
    if (p.copy_err && blockIdx.x == 0) {
        for (int i = threadIdx.x; i < p.T * p.k; i += blockDim.x) {
            p.copy_idx[i] = p.topk_idx[i];
            p.copy_w[i] = p.topk_w[i];
        }
        if (threadIdx.x == 0) *p.copy_err = *reinterpret_cast<const volatile int32_t*>(p.err);
    }
    const int d4 = p.d >> 2;
    const long long total = (long long)p.T * d4;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int t = (int)(i / d4), c = (int)(i - (long long)t * d4);
        float4 acc = p.x ? reinterpret_cast<const float4*>(p.x + (size_t)t * p.d)[c] : make_float4(0.f, 0.f, 0.f, 0.f);
        for (int j = 0; j < p.k; j++) {
            const float w = p.topk_w[t * p.k + j];
            const int pos = p.inv_perm[t * p.k + j];
            const float4 v = reinterpret_cast<const float4*>(p.y + (size_t)pos * p.d)[c];
            acc.x = __fadd_rn(acc.x, __fmul_rn(w, v.x));
            acc.y = __fadd_rn(acc.y, __fmul_rn(w, v.y));
            acc.z = __fadd_rn(acc.z, __fmul_rn(w, v.z));
            acc.w = __fadd_rn(acc.w, __fmul_rn(w, v.w));
        }
        if (p.ys) {
            const float4 v = reinterpret_cast<const float4*>(p.ys + (size_t)t * p.d)[c];
            acc.x = __fadd_rn(acc.x, v.x);
            acc.y = __fadd_rn(acc.y, v.y);
            acc.z = __fadd_rn(acc.z, v.z);
            acc.w = __fadd_rn(acc.w, v.w);
        }
        reinterpret_cast<float4*>(p.out + (size_t)t * p.d)[c] = acc;
    }
}

}  // namespace qrm
