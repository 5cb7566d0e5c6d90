// common.cuh -- shared device helpers and device-side descriptors.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace qrm {

// QuantFormat ids (Dtypes.cs:6-26)
enum Fmt : int32_t {
    F32 = 0, F16 = 1, BF16 = 2, Q4_0 = 3, Q8_0 = 4, Q2_K = 5, Q4_K = 6, Q6_K = 7, TRI = 8,
    I8_BLK = 9, Q3_K = 10, Q5_K = 11, B1 = 12, B1X = 13, T1E = 14, T1E_LO = 15
};

// Dtypes.BlockSpec (Dtypes.cs:38-57)
__host__ __device__ inline bool block_spec(int fmt, int* bs, int* bb) {
    switch (fmt) {
        case F32: *bs = 1; *bb = 4; return true;
        case F16: *bs = 1; *bb = 2; return true;
        case BF16: *bs = 1; *bb = 2; return true;
        case Q4_0: *bs = 32; *bb = 20; return true;
        case Q8_0: *bs = 32; *bb = 34; return true;
        case Q4_K: *bs = 256; *bb = 144; return true;
        case Q6_K: *bs = 256; *bb = 210; return true;
        case TRI: *bs = 64; *bb = 18; return true;
        case Q2_K: *bs = 256; *bb = 84; return true;
        case Q3_K: *bs = 256; *bb = 110; return true;
        case Q5_K: *bs = 256; *bb = 176; return true;
        case I8_BLK: *bs = 256; *bb = 258; return true;
        case B1: *bs = 256; *bb = 34; return true;
        case B1X: *bs = 256; *bb = 47; return true;
        case T1E: *bs = 256; *bb = 40; return true;
        case T1E_LO: *bs = 256; *bb = 32; return true;
        default: return false;
    }
}

// Formats kept in HBM exactly as stored in .qw (no field grouping) and taken
// by the register kernel only: Q2_K, Q3_K, Q5_K, I8_BLK, B1, B1X, T1E, T1E_LO.
inline bool is_raw_fmt(int fmt) {
    return fmt == Q2_K || fmt == Q3_K || fmt == Q5_K || fmt == I8_BLK || fmt == B1 || fmt == B1X || fmt == T1E ||
           fmt == T1E_LO;
}

inline bool is_expert_fmt(int fmt) {
    return fmt == Q4_0 || fmt == Q8_0 || fmt == Q4_K || fmt == Q6_K || fmt == TRI || is_raw_fmt(fmt);
}

// A quantised matrix in HBM.  Q4_K keeps the .qw block bytes unchanged
// (144-byte blocks are 16-byte aligned).  The formats whose blocks are not a
// multiple of 16 bytes are stored with each block's fields grouped by kind
// ("split" layout) so every field is loaded with aligned vector loads; the
// blocks are numbered row-major (row r, block b -> r*blocks_per_row + b):
//   Q4_0: qs[nb][16]  | d[nb] (f16)
//   Q8_0: qs[nb][32]  | d[nb]
//   Q6_K: ql[nb][128] | qh[nb][64] | sc[nb][16] | d[nb]
//   TRI : codes[nb][16] | scale[nb]
// The total size equals the .qw size; no byte value changes.
struct MatDev {
    const uint8_t* base;
    int32_t fmt;
    int32_t rows;
    int32_t cols;
    int32_t pad;
    int64_t nb;  // number of blocks
};

__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}
// Limit of the waits that give up on a stage or a peer that does not deliver
// (producers, consumers, peer flags): 2 s, or QRM_WAIT_LIMIT_US read at layer
// creation.  One copy per translation unit and device; set_wait_limit_here
// sets the calling unit's.  Drains of copies already in flight, which always
// complete, keep a fixed limit.
static __device__ uint64_t g_wait_limit_ns = 2000000000ull;
__device__ __forceinline__ uint64_t wait_limit_ns() { return *reinterpret_cast<volatile uint64_t*>(&g_wait_limit_ns); }
static inline cudaError_t set_wait_limit_here(uint64_t ns) {
    return cudaMemcpyToSymbol(g_wait_limit_ns, &ns, sizeof ns);
}

// Programmatic dependent launch.  A kernel launched with programmatic stream
// serialization may start while its predecessor still runs: pdl_wait() blocks
// until the predecessor grid has completed and its writes are visible (a no-op
// for an ordinary launch); pdl_trigger() lets the successor be scheduled.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Device-side error flag bits, read back by qrm_sync().
enum : uint32_t { ERR_TIMEOUT = 1u, ERR_BOUNDS = 2u, ERR_INTERNAL = 4u };

}  // namespace qrm
