// umma_host.h -- host entry points of the tcgen05 grouped expert path
// (umma.cu), used by the forward in qrmoe.cu.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace qrm {
struct MatDev;

// One work item of the grouped kernel: (expert matrix, row block, block of tokens).
struct UmmaItem {
    int mat;      // index into the matrix table: expert * 3 + which (which = gate for gate/up items)
    int rb;       // row block (64 gate+up rows or 128 down rows)
    int pos;      // first row of the item's tokens in the activation matrix
    int n;        // tokens (1..256)
};

// the grouped kernel's wait limit on the current device (QRM_WAIT_LIMIT_US)
cudaError_t umma_set_wait_limit(uint64_t ns);
// true when matrices of format fmt in the tiled layout can take the path
bool umma_format(int fmt);
// f16 [rows][K] row-major matrix at base as a TMA tensor map (boxes of 64
// columns x 16 rows, 128-byte swizzle); 0 or a CUresult
int umma_encode_map(CUtensorMap* map, const void* base, long long rows, int K);
// f16 activation rows in dispatch order (routed rows: xn rows pos_tok[i],
// then shared_rows rows of xn_shared)
cudaError_t umma_gather(const float* xn, const float* xn_shared, const int32_t* pos_tok, int Tk, int shared_rows, int d,
                        __half* out, int sm_count, cudaStream_t s);
// SwiGLU outputs between the two paths: to_f16 = 1 copies the f32 rows of h
// (routed, [Tk][f]) and hs (shared, [T][f]) into h16 [Tk + T][f]; 0 the reverse
cudaError_t umma_convert_h(float* h, float* hs, int Tk, int shared_rows, int f, __half* h16, int to_f16, int sm_count,
                           cudaStream_t s);
// both stages' work lists from the dispatch's slot table
cudaError_t umma_plan(const int4* slot_info, const int32_t* n_active, int has_shared, int Tk, int rb_gateup,
                      int rb_down, int E, UmmaItem* gu_items, int32_t* gu_count, UmmaItem* dn_items,
                      int32_t* dn_count, int cap, cudaStream_t s);
// routed format fa with shared format fb (-1: no shared expert) has a kernel
bool umma_pair(int fa, int fb);
// the grouped kernel of one stage (gateup: SwiGLU into h_out; else f32 rows);
// items whose rows start at or after shared_pos are the shared expert's (format fb)
cudaError_t umma_expert(int fa, int fb, bool gateup, const CUtensorMap& map, const MatDev* mats, const UmmaItem* items,
                        const int32_t* n_items, int K, int rows, int shared_pos, float limit, __half* h_out,
                        float* y_routed, float* y_shared, int32_t* err, int grid, cudaStream_t s);
// capacity of the work lists for up to Tk routed rows and T shared rows
long long umma_item_cap(int n_local, long long Tk, long long T, int rb_gateup, int rb_down);
constexpr int kUmmaItemBytes = 16;
}  // namespace qrm
