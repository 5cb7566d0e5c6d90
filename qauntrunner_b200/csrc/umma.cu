// umma.cu -- host side of the tcgen05 grouped expert path (umma.cuh): tensor
// maps, the gather and planning kernels, the grouped kernel launches.
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "umma.cuh"
#include "umma_host.h"

namespace qrm {

static_assert(sizeof(UmmaItem) == kUmmaItemBytes, "work item size");

cudaError_t umma_set_wait_limit(uint64_t ns) { return set_wait_limit_here(ns); }

bool umma_format(int fmt) { return fmt == Q4_K || fmt == Q8_0 || fmt == Q4_0 || fmt == Q6_K || fmt == TRI; }

// cuTensorMapEncodeTiled from the driver (no link-time dependency on libcuda)
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static std::once_flag once;
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

int umma_encode_map(CUtensorMap* map, const void* base, long long rows, int K) {
    auto fn = encode_fn();
    if (!fn) return -1;
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    const cuuint32_t box[2] = {64, 16};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return (int)r;
}

cudaError_t umma_gather(const float* xn, const float* xn_shared, const int32_t* pos_tok, int Tk, int shared_rows, int d,
                        __half* out, int sm_count, cudaStream_t s) {
    const long long n = (long long)(Tk + shared_rows) * (d / 8);
    if (n <= 0) return cudaSuccess;
    const int grid = (int)std::min<long long>((n + 255) / 256, (long long)sm_count * 8);
    umma_gather_kernel<<<grid, 256, 0, s>>>(xn, xn_shared, pos_tok, Tk, shared_rows, d, out);
    return cudaGetLastError();
}

__global__ void umma_convert_h_kernel(float* __restrict__ h, float* __restrict__ hs, int Tk, int shared_rows, int f,
                                      __half* __restrict__ h16, int to_f16) {
    const long long n2 = (long long)(Tk + shared_rows) * (f / 2);
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n2; i += (long long)gridDim.x * blockDim.x) {
        const long long row = i / (f / 2);
        const int c = (int)(i - row * (f / 2)) * 2;
        float* src = row < Tk ? h + row * f + c : hs + (row - Tk) * f + c;
        __half2* dst = reinterpret_cast<__half2*>(h16 + row * f + c);
        if (to_f16) {
            *dst = __floats2half2_rn(src[0], src[1]);
        } else {
            const float2 v = __half22float2(*dst);
            src[0] = v.x;
            src[1] = v.y;
        }
    }
}

cudaError_t umma_convert_h(float* h, float* hs, int Tk, int shared_rows, int f, __half* h16, int to_f16, int sm_count,
                           cudaStream_t s) {
    const long long n = (long long)(Tk + shared_rows) * (f / 2);
    if (n <= 0) return cudaSuccess;
    const int grid = (int)std::min<long long>((n + 255) / 256, (long long)sm_count * 8);
    umma_convert_h_kernel<<<grid, 256, 0, s>>>(h, hs, Tk, shared_rows, f, h16, to_f16);
    return cudaGetLastError();
}

cudaError_t umma_plan(const int4* slot_info, const int32_t* n_active, int has_shared, int Tk, int rb_gateup,
                      int rb_down, int E, UmmaItem* gu_items, int32_t* gu_count, UmmaItem* dn_items,
                      int32_t* dn_count, int cap, cudaStream_t s) {
    umma_plan_kernel<<<1, 32, 0, s>>>(slot_info, n_active, has_shared, Tk, rb_gateup, rb_down, E, gu_items, gu_count,
                                      dn_items, dn_count, cap);
    return cudaGetLastError();
}

long long umma_item_cap(int n_local, long long Tk, long long T, int rb_gateup, int rb_down) {
    const long long slots = std::min<long long>(n_local, Tk) + 1;
    const long long blocks = slots + (Tk + T) / kUmmaMaxN + 1;
    return blocks * std::max(rb_gateup, rb_down);
}

template <int FA, int FB, bool GU>
static cudaError_t launch_t(const CUtensorMap& map, const UmmaParams& p, int grid, cudaStream_t s) {
    const UmmaSmem sm = umma_smem(FA, FB);
    // one CTA per SM (it holds all of tensor memory): more than half the shared memory
    if (sm.total <= 114 * 1024 || sm.raw_stages < 2 || sm.b_stages < 2) return cudaErrorInvalidConfiguration;
    static bool attr = false;
    if (!attr) {
        cudaError_t e = cudaFuncSetAttribute(expert_umma_kernel<FA, FB, GU>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm.total);
        if (e != cudaSuccess) return e;
        attr = true;
    }
    expert_umma_kernel<FA, FB, GU><<<grid, kUmmaWarps * 32, sm.total, s>>>(map, p, sm.raw_stages, sm.raw_bytes,
                                                                             sm.b_stages, (int)sm.b_off, (int)sm.x_off);
    return cudaGetLastError();
}

template <int FA, int FB>
static cudaError_t launch_pair(bool gateup, const CUtensorMap& map, const UmmaParams& p, int grid, cudaStream_t s) {
    return gateup ? launch_t<FA, FB, true>(map, p, grid, s) : launch_t<FA, FB, false>(map, p, grid, s);
}

bool umma_pair(int fa, int fb) {
    return (umma_format(fa) && (fb < 0 || fb == fa)) || (fa == Q4_K && fb == Q8_0);
}

cudaError_t umma_expert(int fa, int fb, bool gateup, const CUtensorMap& map, const MatDev* mats,
                        const UmmaItem* items, const int32_t* n_items, int K, int rows, int shared_pos, float limit,
                        __half* h_out, float* y_routed, float* y_shared, int32_t* err, int grid, cudaStream_t s) {
    UmmaParams p{mats, items, n_items, K, rows, shared_pos, limit, h_out, y_routed, y_shared, err};
    if (fb < 0) fb = fa;
    if (fa == Q4_K && fb == Q4_K) return launch_pair<Q4_K, Q4_K>(gateup, map, p, grid, s);
    if (fa == Q4_K && fb == Q8_0) return launch_pair<Q4_K, Q8_0>(gateup, map, p, grid, s);
    if (fa == Q8_0 && fb == Q8_0) return launch_pair<Q8_0, Q8_0>(gateup, map, p, grid, s);
    if (fa == Q4_0 && fb == Q4_0) return launch_pair<Q4_0, Q4_0>(gateup, map, p, grid, s);
    if (fa == Q6_K && fb == Q6_K) return launch_pair<Q6_K, Q6_K>(gateup, map, p, grid, s);
    if (fa == TRI && fb == TRI) return launch_pair<TRI, TRI>(gateup, map, p, grid, s);
    return cudaErrorInvalidValue;
}

}  // namespace qrm
