// layout.cuh -- .qw block bytes <-> device storage layout.
//
// Q4_K blocks (144 B = 9 x 16 B) are stored exactly as in the .qw file.  For
// Q4_0 (20 B), Q8_0 (34 B), Q6_K (210 B) and TRI (18 B) each block's fields
// are grouped by kind so that every field starts on its natural alignment:
//   Q4_0: qs[nb][16] | d[nb][2] | pad[nb][2]   (pad = .qw bytes 18-19, never read)
//   Q8_0: qs[nb][32] | d[nb][2]
//   Q6_K: ql[nb][128] | qh[nb][64] | sc[nb][16] | d[nb][2]
//   TRI : codes[nb][16] | scale[nb][2]
// This is a permutation of bytes: sizes equal the .qw sizes, values are never
// changed, and to_qw reproduces the input exactly.
#pragma once
#include "common.cuh"

namespace qrm {

struct Field { int src_off, len, dst_base_mul; };  // dst = nb*dst_base_mul + blk*len

__device__ __forceinline__ int split_fields(int fmt, Field* f) {
    switch (fmt) {
        case Q4_0: f[0] = {2, 16, 0}; f[1] = {0, 2, 16}; f[2] = {18, 2, 18}; return 3;
        case Q8_0: f[0] = {2, 32, 0}; f[1] = {0, 2, 32}; return 2;
        case Q6_K: f[0] = {0, 128, 0}; f[1] = {128, 64, 128}; f[2] = {192, 16, 192}; f[3] = {208, 2, 208}; return 4;
        case TRI: f[0] = {2, 16, 0}; f[1] = {0, 2, 16}; return 2;
        default: return 0;
    }
}

// to_split = 1: .qw bytes -> split layout; 0: split -> .qw bytes.  One thread
// per (block, byte) pair of the block.
static __global__ void relayout_kernel(int fmt, int bb, const uint8_t* __restrict__ src,
                                uint8_t* __restrict__ dst, long long nb, int to_split) {
    Field f[4];
    const int nf = split_fields(fmt, f);
    const long long total = nb * bb;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const long long blk = i / bb;
        const int byte = (int)(i - blk * bb);
        for (int k = 0; k < nf; k++) {
            if (byte >= f[k].src_off && byte < f[k].src_off + f[k].len) {
                const long long so = nb * f[k].dst_base_mul + blk * f[k].len + (byte - f[k].src_off);
                if (to_split) dst[so] = src[i];
                else dst[i] = src[so];
            }
        }
    }
}

}  // namespace qrm
