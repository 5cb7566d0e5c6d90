// ep.cuh -- expert-parallel data movement.
//
// G ranks, one process per GPU, each holding the routed experts
// [rank*E/G, (rank+1)*E/G) and a replica of norm, router and shared expert.
// Per forward every rank routes its own T tokens; gathered token u = p*T + t
// is rank p's token t on every rank.
//
// Peer-memory mode (NVLink through NVSwitch, the default when every rank can
// map every other rank's memory): each rank owns one "mailbox" allocation,
// mapped into every peer's address space, holding
//   rec_flag[G], out_flag[G]   epoch of the last records / outputs from rank p
//   xn  [G*T][d]               gathered token rows (rows of rank p at p*T)
//   idx [G*T][k]               gathered top-k rows
//   y   [T*k][d]               expert output rows of this rank's tokens
// A sender stores into every rank q the top-k rows of all its tokens and the
// token rows of only those tokens with an expert on q (into its own mailbox
// all of them: the shared expert runs there for the owner's tokens), then
// raises its record flag in q's mailbox.  q's dispatch waits for all G record
// flags and keeps the assignments of its own experts.  After the expert
// stages, each output row (gathered token u = p*T + t, slot j) is stored at
// row t*k + j of owner p's y block -- each assignment has exactly one holder,
// so one block per owner takes every holder's rows -- and the last block of
// the push raises this rank's output flag in every owner's mailbox.  The
// owner's combine waits for all G output flags.  The epoch is a per-rank
// counter in device memory (dispatch advances it), so captured CUDA graphs
// replay correctly.  Every wait is bounded: on expiry the kernel sets
// ERR_TIMEOUT and carries on over the stale (in-bounds) contents; qrm_sync
// reports the error.
//
// Buffer reuse needs no extra handshake: a sender writes forward N+1's
// records into a peer only after its combine of forward N has seen that
// peer's outputs of forward N, which the peer pushed after its expert kernels
// finished reading forward N's records; and it writes forward N+1's outputs
// only after its dispatch has seen the owner's forward N+1 records, which the
// owner sent after its combine of forward N was done with its y block.
//
// NCCL mode: the (token row, top-k indices, top-k weights) records of every
// rank are all-gathered, and output block q ([T*k][d], row t*k+j, only the
// rows of experts this rank holds) goes to owner q by grouped send/recv; the
// owner reads row t*k+j from the block of the rank holding expert idx[t][j].
#pragma once
#include "common.cuh"

namespace qrm {

// Byte offsets inside every rank's mailbox (identical on all ranks).
struct EpMailbox {
    long long rec_flag;   // u32 [G]: epoch of the records received from rank q
    long long out_flag;   // u32 [G]: epoch of the output rows received from rank q
    long long xn;         // f32 [G*T][d] gathered normalised tokens
    long long idx;        // i32 [G*T][k] gathered top-k indices
    long long y;          // f32 [T*k][d] output rows of this rank's tokens (row t*k + j from its holder)
};

struct EpPeers {
    const unsigned long long* base;  // [G] mailbox of each rank, mapped here (own: local)
    EpMailbox mb;
    uint32_t* epoch;      // this rank's forward counter
    uint32_t* cnt;        // [2][G] finished sender blocks per destination (zero between launches)
    int32_t* err;         // ERR_* flags
    int G, rank;
};


__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Waits until *flag has reached `want` (epochs only grow; wrap-safe compare).
// Returns false when the wait gave up (after wait_limit_ns()).
__device__ inline bool ep_wait_flag(const uint32_t* flag, uint32_t want) {
    if ((int32_t)(ld_acquire_sys(flag) - want) >= 0) return true;
    const uint64_t t0 = global_ns(), lim = wait_limit_ns();
    for (int i = 0;; i++) {
        if ((int32_t)(ld_acquire_sys(flag) - want) >= 0) return true;
        if (i >= 256) __nanosleep(256);
        if ((i & 63) == 63 && global_ns() - t0 > lim) return false;
    }
}

// The calling block's stores to rank q are complete: the last of the `nb`
// blocks writing to q raises q's flag `which` (0 records, 1 outputs) for
// this rank to `epoch`.  Cumulative fences order the other blocks' stores
// (observed through the counter) before the flag.
__device__ inline void ep_signal(const EpPeers& p, int which, int q, uint32_t epoch, int nb) {
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        bool last = true;
        if (nb > 1) {
            uint32_t* c = p.cnt + which * p.G + q;
            last = atomicAdd(c, 1u) == (uint32_t)(nb - 1);
            if (last) {
                *c = 0;
                __threadfence_system();
            }
        }
        if (last) {
            char* mb = reinterpret_cast<char*>(p.base[q]);
            uint32_t* flags = reinterpret_cast<uint32_t*>(mb + (which ? p.mb.out_flag : p.mb.rec_flag));
            st_release_sys(flags + p.rank, epoch);
        }
    }
}

// Records of this rank's T tokens into the gathered arrays of every rank q,
// rows [rank*T, rank*T + T): the top-k rows of all T tokens (q's dispatch
// reads them all and keeps the assignments of its own experts), the token
// rows only of tokens with at least one expert on q (epr experts per rank) --
// all of them into this rank's own mailbox, whose rows the shared expert
// reads.  Rows that are not sent are never read.  Grid: G*nb blocks, nb per
// destination.
__global__ void ep_push_records_kernel(const float* __restrict__ xn, const int32_t* __restrict__ idx, int T, int d,
                                       int k, int epr, EpPeers p) {
    const int nb = gridDim.x / p.G, q = blockIdx.x / nb, part = blockIdx.x - q * nb;
    const uint32_t epoch = *p.epoch + 1;
    char* mb = reinterpret_cast<char*>(p.base[q]);
    const int d4 = d / 4;
    int32_t* di = reinterpret_cast<int32_t*>(mb + p.mb.idx) + (size_t)p.rank * T * k;
    for (int i = part * blockDim.x + threadIdx.x; i < T * k; i += nb * blockDim.x) di[i] = idx[i];
    float4* dx = reinterpret_cast<float4*>(mb + p.mb.xn) + (size_t)p.rank * T * d4;
    const float4* sx = reinterpret_cast<const float4*>(xn);
    const bool own = q == p.rank;
    int t_seen = -1;
    bool need = false;
    for (long long i = part * (long long)blockDim.x + threadIdx.x; i < (long long)T * d4; i += (long long)nb * blockDim.x) {
        const int t = (int)(i / d4);
        if (t != t_seen) {
            t_seen = t;
            need = own;
            for (int j = 0; j < k && !need; j++) need = idx[t * k + j] / epr == q;
        }
        if (need) dx[i] = sx[i];
    }
    ep_signal(p, 0, q, epoch, nb);
}

// Output rows of the local experts straight into the owners' receive blocks:
// position pos < n_pos of the dispatch holds assignment a = perm[pos] =
// u*k + j of gathered token u = q*T + t (owner q, its token t), and its row
// goes to row t*k + j of owner q's block.  Each assignment has exactly one
// holder, so one [T*k][d] block per owner takes every holder's rows.  Once
// every block has stored its rows, the last one raises this rank's output
// flag in every owner's mailbox (also those that get no rows: the flags
// count forwards).
__global__ void ep_push_outputs_kernel(const float* __restrict__ y, const int32_t* __restrict__ perm,
                                       const int32_t* __restrict__ n_pos, int T, int k, int d, EpPeers p) {
    const uint32_t epoch = *p.epoch;   // advanced by this forward's dispatch
    const int d4 = d / 4;
    const long long n = (long long)(*n_pos) * d4;
    const float4* src = reinterpret_cast<const float4*>(y);
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const int pos = (int)(i / d4), c = (int)(i - (long long)pos * d4);
        const int a = perm[pos], u = a / k, j = a - u * k, q = u / T, t = u - q * T;
        char* mb = reinterpret_cast<char*>(p.base[q]);
        reinterpret_cast<float4*>(mb + p.mb.y)[((size_t)t * k + j) * d4 + c] = src[i];
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        uint32_t* c = p.cnt + p.G;   // output counter
        if (atomicAdd(c, 1u) == gridDim.x - 1) {
            *c = 0;
            __threadfence_system();
            for (int q = 0; q < p.G; q++) {
                char* mb = reinterpret_cast<char*>(p.base[q]);
                st_release_sys(reinterpret_cast<uint32_t*>(mb + p.mb.out_flag) + p.rank, epoch);
            }
        }
    }
}

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
// (combine_kernel's arithmetic).  recv holds row t*k + j of y_j: in one
// [T*k][d] block (peer memory), or per holder ([G][T*k][d], NCCL; the block
// of the rank that holds expert idx[t][j], epr experts per rank).
// In peer-memory mode (`wait_flags` set) every block first waits for the
// output flags of all G holders.
__global__ void ep_combine_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                  const int32_t* __restrict__ idx, const float* __restrict__ recv,
                                  const float* __restrict__ ys, int T, int k, int d, int epr, int per_holder,
                                  float* __restrict__ out, const uint32_t* wait_flags, const uint32_t* epoch, int G,
                                  int32_t* err) {
    if (wait_flags) {
        const uint32_t want = *epoch;
        if ((int)threadIdx.x < G && !ep_wait_flag(wait_flags + threadIdx.x, want)) atomicOr(err, (int32_t)ERR_TIMEOUT);
        __syncthreads();
    }
    const int d4 = d / 4;
    const long long total = (long long)T * d4;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int t = (int)(i / d4), c = (int)(i - (long long)t * d4);
        float4 acc = x ? reinterpret_cast<const float4*>(x + (size_t)t * d)[c] : make_float4(0.f, 0.f, 0.f, 0.f);
        for (int j = 0; j < k; j++) {
            const float wj = w[t * k + j];
            const size_t q = per_holder ? (size_t)(idx[t * k + j] / epr) : 0;
            const float4 v = reinterpret_cast<const float4*>(recv + ((q * T + t) * k + j) * d)[c];
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
