// gemv_stream.cuh -- decode-size expert products on the integer tensor cores,
// streamed from a tiled weight layout.
//
// Tiled layout.  A matrix taken by this kernel (Q4_K, Q8_0 or Q4_0; columns a
// multiple of 256; rows a multiple of 8) is stored in HBM as 8-row tiles, and
// each tile as its super-blocks (256 columns) in order.  The chunk of one tile
// and one super-block holds the same bytes as the 8 rows' blocks of that
// super-block, grouped so that the tensor-core fragment loads of a warp read
// consecutive bytes:
//   Q4_K (1152 B): hdr[8 rows][16]  (d, dmin, scales: block bytes 0-15)
//                  qs[4 pairs][8 rows][32]  (block bytes 16 + 32*pair ...)
//   Q8_0 (2176 B): d[8 rows][8 blocks][2]  qs[8 blocks][8 rows][32]
//   Q4_0 (1280 B): d[8 rows][8 blocks][2]  pad[8 rows][8 blocks][2]
//                  qs[8 blocks][8 rows][16]
// The chunks of a tile are consecutive, so a K range of a tile is one run of
// bytes: a stage (16 or 32 MMA rows x a K range) is filled by one bulk copy
// per 8-row tile run, and the shared-memory image is the HBM image (no row
// padding, no bank conflicts).  This is a permutation of the .qw bytes (sizes
// and values unchanged); tiled_offset() maps every byte both ways.
//
// Kernel.  An item is (segment, expert slot, row group); its K range is split
// into `parts` stages of `sbs` super-blocks, streamed through a ring of S
// stages by one producer warp.  The CW consumer warps split each stage into
// units of (16-row MMA tile, super-block, half = groups 0-3 or 4-7); a unit is
// four mma.sync m16n8k32 per token on the raw codes against the 16-bit
// fixed-point activation tables (gemv_imma.cuh), the per-group scales applied
// in f32.  A stage is released as soon as its units are done; after the last
// part each warp publishes its partial sums to a reduction slot, and the last
// warp to publish adds the CW partials in a fixed order (SwiGLU for gate/up).
// Tokens: passes of NTK tokens, stream_passes(NTK) passes per item chunk; an
// expert slot with more tokens streams its weights once per chunk of
// stream_chunk(NTK) tokens (one token per chunk when T = 1).  All waits are bounded.
#pragma once
#include <algorithm>
#include <cstdlib>

#include "common.cuh"
#include "gemv.cuh"
#include "gemv_imma.cuh"
#include "gemv_tma.cuh"

namespace qrm {

// ------------------------------------------------------------ tiled layout

// bytes of one row's blocks in one super-block (256 columns)
__host__ __device__ inline int tile_row_sb_bytes(int fmt) {
    switch (fmt) {
        case Q4_K: return 144;
        case Q8_0: return 272;
        case Q4_0: return 160;
        case Q6_K: return 210;
        case TRI: return 72;
        default: return 0;
    }
}
__host__ __device__ inline int tile_chunk_bytes(int fmt) { return 8 * tile_row_sb_bytes(fmt); }

// Offset in the tiled matrix of byte `byte` of block `blk` (.qw order: row
// major, `nsb` super-blocks per row).  Chunk layouts (8 rows r, one super-block):
//   Q4_K hdr[r][16] | qs[pair][r][32]          Q8_0 d[r][blk][2] | qs[blk][r][32]
//   Q4_0 d[r][blk][2] | pad[r][blk][2] | qs[blk][r][16]
//   Q6_K ql[r][128] | qh[r][64] | sc[r][16] | d[r][2]
//   TRI  codes[r][blk][16] | scale[r][blk][2]   (4 blocks of 64 weights)
__host__ __device__ inline long long tiled_offset(int fmt, int nsb, long long blk, int byte) {
    const int bps = (fmt == Q4_K || fmt == Q6_K) ? 1 : fmt == TRI ? 4 : 8;   // blocks per super-block
    const long long bpr = (long long)nsb * bps;    // blocks per row
    const long long row = blk / bpr;
    const int b = (int)(blk - row * bpr), sb = b / bps, g = b - sb * bps;
    const long long rt = row >> 3;
    const int r = (int)(row & 7);
    const long long chunk = (rt * nsb + sb) * (long long)tile_chunk_bytes(fmt);
    switch (fmt) {
        case Q4_K:
            if (byte < 16) return chunk + 16 * r + byte;
            return chunk + 128 + 256 * ((byte - 16) >> 5) + 32 * r + ((byte - 16) & 31);
        case Q8_0:
            if (byte < 2) return chunk + 16 * r + 2 * g + byte;
            return chunk + 128 + 256 * g + 32 * r + (byte - 2);
        case Q6_K:   // ql (0-127), qh (128-191), scales (192-207), d (208-209)
            if (byte < 128) return chunk + 128 * r + byte;
            if (byte < 192) return chunk + 1024 + 64 * r + (byte - 128);
            if (byte < 208) return chunk + 1536 + 16 * r + (byte - 192);
            return chunk + 1664 + 2 * r + (byte - 208);
        case TRI:    // scale (0-1), codes (2-17)
            if (byte < 2) return chunk + 512 + 8 * r + 2 * g + byte;
            return chunk + 64 * r + 16 * g + (byte - 2);
        default:  // Q4_0: d (0-1), qs (2-17), pad (18-19)
            if (byte < 2) return chunk + 16 * r + 2 * g + byte;
            if (byte >= 18) return chunk + 128 + 16 * r + 2 * g + (byte - 18);
            return chunk + 256 + 128 * g + 16 * r + (byte - 2);
    }
}

// to_tiled = 1: .qw bytes -> tiled; 0: tiled -> .qw bytes.  One thread per byte.
static __global__ void tile_relayout_kernel(int fmt, int bb, int nsb, const uint8_t* __restrict__ src,
                                     uint8_t* __restrict__ dst, long long nb, int to_tiled) {
    const long long total = nb * bb;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const long long blk = i / bb;
        const int byte = (int)(i - blk * bb);
        const long long t = tiled_offset(fmt, nsb, blk, byte);
        if (to_tiled) dst[t] = src[i];
        else dst[i] = src[t];
    }
}

// ------------------------------------------------------------ stage plan

constexpr int kStreamMaxStages = 16;
constexpr int kStreamMaxWarps = 16;            // consumer warps, one token per pass
constexpr int kStreamMaxWarps2 = 14;           // two tokens per pass
constexpr int kStreamPasses1 = 1;              // passes per item chunk, one token per pass (T = 1)
constexpr int kStreamPasses2 = 2;              // two tokens per pass
constexpr int kStreamMaxR16 = 2;               // most 16-row MMA tiles per gate/up item
constexpr int kStreamMaxR16Down = 4;           // most 16-row MMA tiles per down item
constexpr int kStreamRedSlots = 4;
constexpr int kStreamMaxChunk = 4;             // most tokens per item chunk
// per-stage header: item, slot, e, off, chunk tokens, seg, part, row group,
// first token of the chunk, table rows of the chunk's tokens
constexpr int kStreamHdrInts = 16;
constexpr int kStreamCtlOff = 8 * (2 * kStreamMaxStages + 1);   // after full[], empty[], the table barrier
constexpr int kStreamHdrOff = 512;
// the producer's table of this CTA's next items (resolved 32 at a time)
constexpr int kStreamItemBatch = 32;
constexpr int kStreamItemBytes = 32;
constexpr int kStreamItemOff = kStreamHdrOff + kStreamMaxStages * kStreamHdrInts * 4;
constexpr int kStreamDataOff = (kStreamItemOff + kStreamItemBatch * kStreamItemBytes + 127) / 128 * 128;
static_assert(kStreamCtlOff + 48 <= kStreamHdrOff, "stream control area: abort flag, arrivals, tickets");

__host__ __device__ constexpr int stream_passes(int ntk) { return ntk == 1 ? kStreamPasses1 : kStreamPasses2; }
// tokens per item chunk
__host__ __device__ constexpr int stream_chunk(int ntk) { return ntk * stream_passes(ntk); }
static_assert(stream_chunk(1) <= kStreamMaxChunk && stream_chunk(2) <= kStreamMaxChunk, "header table rows");

struct StreamSeg {
    int fmt;           // -1: no such segment in the launch
    int r16;           // 16-row MMA tiles per item
    int halves;        // 1: a unit is a super-block; 2: half of one
    int sbs;           // super-blocks per stage
    int parts;         // stages per item (K range / sbs)
    int cb;            // bytes of one tile chunk (8 rows x 1 super-block)
    int stage_bytes;   // weight bytes of one stage
    int items_per_slot;
};

struct StreamConfig {
    StreamSeg seg[2];
    int stages;
    int stage_bytes;   // ring slot size (the larger segment)
    int xtab_bytes;    // per token table (16-byte multiple)
    int res_rows;      // > 0: all table rows resident in shared memory; 0: tables read from global
    int red_bytes;     // one reduction slot: [CW][red_tok][16] floats
    int red_tok;       // tokens per reduction slot: min(chunk tokens, tokens of the launch)
    int cw;            // consumer warps
};

// Most 16-row MMA tiles per item: 2 for gate/up (the item then spans the whole
// d_model in two 64 KB stages); 4 for down, whose rows are short (d_ff): a
// 64-row item spans two stages, so the per-item reduction and hand-over come
// once per two stages instead of once per stage.  QRM_STREAM_DOWN_R16
// overrides the down cap for tuning runs.
__host__ inline int stream_max_r16(int M) {
    if (M == 2) return kStreamMaxR16;
    static int v = -1;
    if (v < 0) {
        const char* e = getenv("QRM_STREAM_DOWN_R16");
        v = e ? std::max(1, std::min(kStreamMaxR16Down, atoi(e))) : kStreamMaxR16Down;
    }
    return v;
}

// Segment geometry for `cw` consumer warps.  Every warp keeps one MMA tile
// of the item (cw / r16 warps per tile) and takes the same number of units
// of it per stage; a unit is one super-block (halves = 1) or one half of one
// (groups 0-3 or 4-7, halves = 2).  Chosen: the most MMA tiles per item
// (r16 <= max_r16, dividing the rows and cw), then whole
// super-blocks before halves, then the most super-blocks per stage (dividing
// the row) within `target` bytes.
__host__ inline bool stream_seg(int fmt, int M, int rows, int cols, int target, int cw, int max_r16, StreamSeg* g) {
    *g = StreamSeg{};
    g->fmt = fmt;
    if (fmt < 0) return true;
    const int cb = tile_chunk_bytes(fmt);
    if (!cb || cols % 256) return false;
    const int nsb = cols / 256;
    const int rows_per_mma = M == 2 ? 8 : 16;   // matrix rows per MMA tile
    for (int r16 = max_r16; r16 >= 1; r16--) {
        if (rows % (rows_per_mma * r16) || cw % r16) continue;
        const int wpt = cw / r16;   // warps per MMA tile
        for (int halves = 1; halves <= 2; halves++) {
            for (int sbs = nsb; sbs >= 1; sbs--) {
                if (nsb % sbs || (sbs * halves) % wpt) continue;
                const int bytes = 2 * r16 * sbs * cb;
                if (bytes > target) continue;
                g->r16 = r16;
                g->halves = halves;
                g->sbs = sbs;
                g->parts = nsb / sbs;
                g->cb = cb;
                g->stage_bytes = bytes;
                g->items_per_slot = rows / (rows_per_mma * r16);
                return true;
            }
        }
    }
    return false;
}

// The target stage size (bytes): 64 KB for gate/up; 80 KB for down, where a
// 64-row item of a d_ff = 2048 Q4_K matrix (73.7 KB) then fills one stage
// (two stages fit beside the resident tables; measured at C5 T = 4 / 16:
// down 120 -> 107 us / 365 -> 325 us against two 36.9 KB stages per item).
// QRM_STREAM_STAGE_KB overrides both for tuning runs.
__host__ inline int stream_target_bytes(int M) {
    static int v = -1;
    if (v < 0) {
        const char* e = getenv("QRM_STREAM_STAGE_KB");
        v = e ? std::max(4, atoi(e)) * 1024 : 0;
    }
    return v > 0 ? v : (M == 2 ? 64 : 80) * 1024;
}

// Tables stay resident in shared memory (quantised by the consumers while the
// first stages stream in) when that leaves this many stages, or as many as
// without them.  Two: a separate table launch before the stage costs more
// than the third stage gains (C5 decode down 37.0 -> 32.9 us with two 73.7 KB
// stages and resident tables; T = 4 gate/up 155 -> 142 us).
// QRM_STREAM_RES_MIN overrides it for tuning runs.
__host__ inline int stream_res_min_stages() {
    static int v = -1;
    if (v < 0) {
        const char* e = getenv("QRM_STREAM_RES_MIN");
        v = e ? std::max(2, atoi(e)) : 2;
    }
    return v;
}

// fmt[0] / fmt[1]: formats of the routed and the shared segment (-1: none).
// Consumer warps: among the counts (up to the register budget of NTK) for
// which every segment has a balanced geometry, 12 or more warps first (they
// hide the MMA and shared-load latencies), then the most segments on whole
// super-block units, then the most warps (QRM_STREAM_CW forces a count for
// tuning runs).  max_tok = the most tokens of one expert slot (the launch's
// tokens).  max_r16 = the most MMA tiles per item (stream_max_r16, or fewer
// when the launch has few items).  tab_rows = table rows the launch reads;
// they are kept resident when that leaves stream_res_min_stages() stages,
// else read from global memory.
__host__ inline bool stream_plan(const int (&fmt)[2], int M, int rows, int cols, int ntk, int tab_rows, int max_tok,
                                 int smem_budget, int max_r16, StreamConfig* c) {
    if (fmt[0] < 0 && fmt[1] < 0) return false;
    const int target = stream_target_bytes(M);
    static int forced = -1;
    if (forced < 0) {
        const char* e = getenv("QRM_STREAM_CW");
        forced = e ? std::max(0, atoi(e)) : 0;
    }
    const int max_w = ntk == 1 ? kStreamMaxWarps : kStreamMaxWarps2;
    int best = -1;
    for (int cw = max_w; cw >= 1; cw--) {
        if (forced > 0 && forced <= max_w && cw != forced) continue;
        StreamSeg sg[2];
        bool ok = true;
        int full = 0;
        for (int i = 0; i < 2; i++) {
            if (!stream_seg(fmt[i], M, rows, cols, target, cw, max_r16, &sg[i])) ok = false;
            else if (fmt[i] >= 0 && sg[i].halves == 1) full++;
        }
        const int score = (cw >= 12 ? 1000 : 0) + 100 * full + cw;
        if (!ok || score <= best) continue;
        best = score;
        c->cw = cw;
        c->seg[0] = sg[0];
        c->seg[1] = sg[1];
    }
    if (best < 0) return false;
    c->stage_bytes = 0;
    for (int i = 0; i < 2; i++)
        if (fmt[i] >= 0) c->stage_bytes = std::max(c->stage_bytes, c->seg[i].stage_bytes);
    c->xtab_bytes = xtab_stride(cols);
    c->red_tok = std::max(1, std::min(stream_chunk(ntk), max_tok));
    c->red_bytes = c->cw * c->red_tok * 16 * 4;
    const long long avail = (long long)smem_budget - kStreamDataOff - (long long)kStreamRedSlots * c->red_bytes;
    const long long res = (long long)tab_rows * c->xtab_bytes;
    long long s_res = res < avail ? (avail - res) / c->stage_bytes : 0;
    long long s_glb = avail / c->stage_bytes;
    s_res = std::min<long long>(s_res, kStreamMaxStages);
    s_glb = std::min<long long>(s_glb, kStreamMaxStages);
    if (tab_rows > 0 && s_res >= std::min<long long>(stream_res_min_stages(), s_glb)) {
        c->res_rows = tab_rows;
        c->stages = (int)s_res;
    } else {
        c->res_rows = 0;
        c->stages = (int)s_glb;
    }
    return c->stages >= 2;
}

inline size_t stream_smem_bytes(const StreamConfig& c) {
    return (size_t)kStreamDataOff + (size_t)c.res_rows * c.xtab_bytes + (size_t)kStreamRedSlots * c.red_bytes +
           (size_t)c.stages * c.stage_bytes;
}

// ------------------------------------------------------------ one unit

// Adds to y[q][0] / y[q][1] (rows gid / gid+8 of the MMA tile; this lane's
// groups t and t+4 when FULL, else group 4*half + t) the products of
// super-block sbg (of the row) for nt <= NTK tokens: all eight groups (FULL)
// or the four of `half`.  cA / cB: shared addresses of the super-block's
// chunks of the tile's first / second 8 rows.  Group g's MMAs accumulate into
// chain g / 4 (two independent chains when FULL).
template <int FMT, int NTK, bool SM, bool FULL>
__device__ __forceinline__ void stream_unit(const uint8_t* cA, const uint8_t* cB, const typename TabLd<SM>::Ptr (&tq)[NTK], int nt,
                                            int K, int sbg, int half, int lane, const uint32_t (&bm)[4],
                                            float (&y)[NTK][2]) {
    using L = TabLd<SM>;
    constexpr int NH = FULL ? 2 : 1;   // group halves in this unit
    constexpr int NW = FMT == Q8_0 ? 8 : 4;   // code words per half and group pair
    const int gid = lane >> 2, t = lane & 3, j = gid >> 1, hl = gid & 1;
    const uint32_t sA = smem_u32(cA), sB = smem_u32(cB);
    // every shared load of the unit first (in this order), then the MMAs and
    // the epilogue: B bytes of group 4*h + j (this lane's part of the fixed
    // point), the codes, the scales, the table scale/sum entries
    const int bo = hl * xtab_lo(K) + 32 * j + (FMT == Q4_0 ? 4 : 8) * t + 256 * sbg;
    uint32_t bx[NH][NTK][2];
#pragma unroll
    for (int hh = 0; hh < NH; hh++) {
        const int o = bo + 128 * (FULL ? hh : half);
#pragma unroll
        for (int q = 0; q < NTK; q++) {
            if (q == 0 || q < nt) {
                if (FMT == Q4_0) {
                    bx[hh][q][0] = L::ld32(tq[q], o);
                    bx[hh][q][1] = L::ld32(tq[q], o + 16);
                } else {
                    const uint2 a = L::ld64(tq[q], o);
                    bx[hh][q][0] = a.x;
                    bx[hh][q][1] = a.y;
                }
            } else {
                bx[hh][q][0] = bx[hh][q][1] = 0u;
            }
        }
    }
    uint32_t w[NH][2][NW];   // [half][group pair][words of rows gid, gid+8]
#pragma unroll
    for (int hh = 0; hh < NH; hh++) {
#pragma unroll
        for (int pp = 0; pp < 2; pp++) {
            const int pr = 2 * (FULL ? hh : half) + pp;   // groups 2pr, 2pr+1
            uint32_t* ww = w[hh][pp];
            if (FMT == Q4_K) {
                const uint32_t o = 128 + 256 * pr + 32 * gid + 8 * t;
                const uint2 w0 = lds64(sA + o), w1 = lds64(sB + o);
                ww[0] = w0.x; ww[1] = w0.y; ww[2] = w1.x; ww[3] = w1.y;
            } else if (FMT == Q8_0) {
                const uint32_t o = 128 + 256 * (2 * pr) + 32 * gid + 8 * t;
                const uint2 a0 = lds64(sA + o), a1 = lds64(sB + o);
                const uint2 b0 = lds64(sA + o + 256), b1 = lds64(sB + o + 256);
                ww[0] = a0.x; ww[1] = a0.y; ww[2] = a1.x; ww[3] = a1.y;
                ww[4] = b0.x; ww[5] = b0.y; ww[6] = b1.x; ww[7] = b1.y;
            } else {  // Q4_0
                const uint32_t o = 256 + 128 * (2 * pr) + 16 * gid + 4 * t;
                ww[0] = lds32(sA + o); ww[1] = lds32(sB + o);
                ww[2] = lds32(sA + o + 128); ww[3] = lds32(sB + o + 128);
            }
        }
    }
    uint4 hd[2];             // Q4_K block headers of rows gid, gid+8
    uint32_t dd[NH][2];      // Q8_0 / Q4_0: d of rows gid, gid+8 per half
    if (FMT == Q4_K) {
        hd[0] = lds128(sA + 16 * gid);
        hd[1] = lds128(sB + 16 * gid);
    } else {
#pragma unroll
        for (int hh = 0; hh < NH; hh++) {
            const uint32_t o = 16 * gid + 2 * (t + 4 * (FULL ? hh : half));
            dd[hh][0] = lds16(sA + o);
            dd[hh][1] = lds16(sB + o);
        }
    }
    uint2 ss[NH][NTK];
#pragma unroll
    for (int hh = 0; hh < NH; hh++) {
        const int so = xtab_ss(K) + 8 * (8 * sbg + 4 * (FULL ? hh : half) + t);
#pragma unroll
        for (int q = 0; q < NTK; q++) ss[hh][q] = (q == 0 || q < nt) ? L::ld64(tq[q], so) : make_uint2(0u, 0u);
    }
    // MMAs: group pairs (2pr, 2pr+1) of each half, the halves' chains interleaved
    int X[NH][NTK][4];
#pragma unroll
    for (int hh = 0; hh < NH; hh++)
#pragma unroll
        for (int q = 0; q < NTK; q++)
#pragma unroll
            for (int i = 0; i < 4; i++) X[hh][q][i] = 0;
#pragma unroll
    for (int pp = 0; pp < 2; pp++) {
        uint32_t A0[NH][4], A1[NH][4];
#pragma unroll
        for (int hh = 0; hh < NH; hh++) {
            const uint32_t* ww = w[hh][pp];
            if (FMT == Q4_K) {
                A0[hh][0] = ww[0] & 0x0F0F0F0Fu; A0[hh][1] = ww[2] & 0x0F0F0F0Fu;
                A0[hh][2] = ww[1] & 0x0F0F0F0Fu; A0[hh][3] = ww[3] & 0x0F0F0F0Fu;
                A1[hh][0] = ww[0] & 0xF0F0F0F0u; A1[hh][1] = ww[2] & 0xF0F0F0F0u;
                A1[hh][2] = ww[1] & 0xF0F0F0F0u; A1[hh][3] = ww[3] & 0xF0F0F0F0u;
            } else if (FMT == Q8_0) {
                A0[hh][0] = ww[0]; A0[hh][1] = ww[2]; A0[hh][2] = ww[1]; A0[hh][3] = ww[3];
                A1[hh][0] = ww[4]; A1[hh][1] = ww[6]; A1[hh][2] = ww[5]; A1[hh][3] = ww[7];
            } else {  // Q4_0: low nibbles = weights 0-15 of the block, high = 16-31
                A0[hh][0] = ww[0] & 0x0F0F0F0Fu; A0[hh][1] = ww[1] & 0x0F0F0F0Fu;
                A0[hh][2] = (ww[0] >> 4) & 0x0F0F0F0Fu; A0[hh][3] = (ww[1] >> 4) & 0x0F0F0F0Fu;
                A1[hh][0] = ww[2] & 0x0F0F0F0Fu; A1[hh][1] = ww[3] & 0x0F0F0F0Fu;
                A1[hh][2] = (ww[2] >> 4) & 0x0F0F0F0Fu; A1[hh][3] = (ww[3] >> 4) & 0x0F0F0F0Fu;
            }
        }
#pragma unroll
        for (int g2 = 0; g2 < 2; g2++) {
            const int gm = 2 * pp + g2;   // column pair of the group within its half
#pragma unroll
            for (int hh = 0; hh < NH; hh++) {
                const uint32_t(&A)[4] = g2 ? A1[hh] : A0[hh];
#pragma unroll
                for (int q = 0; q < NTK; q++) {
                    const uint32_t b0 = bx[hh][q][0] & bm[gm], b1 = bx[hh][q][1] & bm[gm];
                    if (FMT == Q8_0) mma_s8s8(X[hh][q], A, b0, b1);
                    else mma_u8s8(X[hh][q], A, b0, b1);
                }
            }
        }
    }
    // scales of group 4*h + t for rows gid (A) and gid+8 (B): y += a*c*s - m*sum
    float ar[NH][2], mr[NH][2];
    if (FMT == Q4_K) {
        // Q4_K: odd groups (high nibbles) keep the nibble in place (code * 16)
        const float kq = (t & 1) ? 4.f : 64.f;
        const uint32_t sel = 0x7044u | ((uint32_t)t << 8);   // byte t -> bits 16..23 of 2.0f
#pragma unroll
        for (int rw = 0; rw < 2; rw++) {
            const uint4 h4 = hd[rw];
            const float d = h2f((uint16_t)(h4.x & 0xFFFF)), dmin = h2f((uint16_t)(h4.x >> 16));
            const float da = kq * d, db = -2.f * kq * d, ma = 64.f * dmin, mb = -128.f * dmin;
            // GetScaleMinK4 (BlockDequantizer.cs:155-166), four sub-blocks per word:
            // sc[0..3] = q[0..3] & 63, m[0..3] = q[4..7] & 63,
            // sc[4..7] = (q[8..11] & 15) | (q[0..3] >> 6) << 4, m[4..7] = (q[8..11] >> 4) | (q[4..7] >> 6) << 4
#pragma unroll
            for (int hh = 0; hh < NH; hh++) {
                const int h = FULL ? hh : half;
                const uint32_t SC = h ? ((h4.w & 0x0F0F0F0Fu) | ((h4.y >> 2) & 0x30303030u)) : (h4.y & 0x3F3F3F3Fu);
                const uint32_t MN = h ? (((h4.w >> 4) & 0x0F0F0F0Fu) | ((h4.z >> 2) & 0x30303030u)) : (h4.z & 0x3F3F3F3Fu);
                // byte b at bits 16..23 of 2.0f reads 2 + b/64: d*b = F*64d - 128d (the
                // high-nibble groups take another 1/16)
                ar[hh][rw] = fmaf(__uint_as_float(prmt(SC, 0x40000000u, sel)), da, db);
                mr[hh][rw] = fmaf(__uint_as_float(prmt(MN, 0x40000000u, sel)), ma, mb);
            }
        }
    } else {
#pragma unroll
        for (int hh = 0; hh < NH; hh++) {
            const float dA = h2f((uint16_t)dd[hh][0]), dB = h2f((uint16_t)dd[hh][1]);
            ar[hh][0] = dA;
            ar[hh][1] = dB;
            mr[hh][0] = FMT == Q4_0 ? 8.f * dA : 0.f;
            mr[hh][1] = FMT == Q4_0 ? 8.f * dB : 0.f;
        }
    }
#pragma unroll
    for (int hh = 0; hh < NH; hh++) {
#pragma unroll
        for (int q = 0; q < NTK; q++) {
            if (q == 0 || q < nt) {
                const float scl = __uint_as_float(ss[hh][q].x), sum = __uint_as_float(ss[hh][q].y);
                const float c0 = (float)(X[hh][q][0] * 256 + X[hh][q][1]), c1 = (float)(X[hh][q][2] * 256 + X[hh][q][3]);
                float a = y[q][0], b = y[q][1];
                a = fmaf(ar[hh][0], c0 * scl, a);
                b = fmaf(ar[hh][1], c1 * scl, b);
                if (FMT != Q8_0) {
                    a = fmaf(-mr[hh][0], sum, a);
                    b = fmaf(-mr[hh][1], sum, b);
                }
                y[q][0] = a;
                y[q][1] = b;
            }
        }
    }
}

// ------------------------------------------------------------ reductions
struct StreamRed {
    int* arr;     // [slots] warps arrived with their partials
    int* tick;    // [slots] reductions completed in the slot
    float* buf;   // [slots][red floats]
    int floats;   // floats per slot
};

// What a reduction needs once the stages and their headers are gone.
struct StreamJob {
    int r;         // reduction number (slot r % kStreamRedSlots)
    int seg, rg, off, t0, nt, shared;
};

// The reduction of job j (all CW warps' partials are in its slot): adds the
// partials of each MMA tile's warps in a fixed order, applies SwiGLU
// (gate/up) and writes the outputs; frees the slot.  Partials: [CW][chunk
// tokens][16], warp w holding MMA tile w / (CW / r16); rows 0-7 = gate, 8-15
// = up (M = 2) or 16 consecutive rows (M = 1).  Run by one warp.
template <int M, int NTK>
__device__ __forceinline__ void stream_reduce(const GemvParams& p, const StreamConfig& cfg, const StreamJob& j,
                                              const StreamRed& R, int lane) {
    constexpr int OUT = M == 2 ? 8 : 16;   // outputs per MMA tile and token
    const int r16 = j.seg ? cfg.seg[1].r16 : cfg.seg[0].r16, wpt = cfg.cw / r16;
    const int sq = j.r % kStreamRedSlots;
    const float* red = R.buf + (size_t)sq * R.floats;
    __threadfence_block();
    for (int o = lane; o < r16 * j.nt * OUT; o += 32) {
        const int i = o / (j.nt * OUT), rem = o - i * (j.nt * OUT), q = rem / OUT, r = rem - q * OUT;
        float v[M];
#pragma unroll
        for (int m = 0; m < M; m++) {
            float sum = 0.f;
            for (int w = i * wpt; w < (i + 1) * wpt; w++) sum += red[(w * cfg.red_tok + q) * 16 + m * 8 + r];
            v[m] = sum;
        }
        const float res = M == 2 ? swiglu(v[0], v[M - 1], p.limit) : v[0];
        const int tk = j.t0 + q;
        float* orow = j.shared ? p.out_shared + (size_t)tk * p.rows : p.out_routed + (size_t)(j.off + tk) * p.rows;
        if (M == 1 && p.ep_base && !j.shared) {
            // the owner's row of this assignment (a = u*k + s, u = owner*T + t)
            const int a = p.perm[j.off + tk], u = a / p.k, s = a - u * p.k, own = u / p.ep_T, t = u - own * p.ep_T;
            orow = reinterpret_cast<float*>(reinterpret_cast<char*>(p.ep_base[own]) + p.ep_y) + ((size_t)t * p.k + s) * p.rows;
        }
        orow[(j.rg * r16 + i) * OUT + r] = res;
    }
    __syncwarp();
    if (lane == 0) {
        R.arr[sq] = 0;
        __threadfence_block();
        *reinterpret_cast<volatile int*>(&R.tick[sq]) = j.r / kStreamRedSlots + 1;
    }
}

// ------------------------------------------------------------ one stage
// This warp's units of one stage (format FMT), accumulated into y: MMA tile
// w / wpt, units w % wpt + n * wpt (n < sbs * halves / wpt).
template <int FMT, int M, int NTK>
__device__ __forceinline__ void stream_stage(const GemvParams& p, const StreamConfig& cfg, const StreamSeg& g,
                                             const int* h, const uint8_t* st, const uint8_t* res, int warp, int lane,
                                             const uint32_t (&bm)[4], float (&y)[stream_passes(NTK)][NTK][2]) {
    constexpr int P = stream_passes(NTK);
    const int K = p.cols, nc = h[4], part = h[6];
    const int res_bytes = cfg.res_rows * cfg.xtab_bytes;
    const int wpt = cfg.cw / g.r16, i = warp / wpt, wt = warp - i * wpt;
    // shared-memory chunks of MMA tile i: gate/up stage = [gate tiles][up tiles],
    // down stage = consecutive 8-row tiles
    const int ta = M == 2 ? i : 2 * i, tb = M == 2 ? g.r16 + i : 2 * i + 1;
    const int nu = g.sbs * g.halves;
    for (int u = wt; u < nu; u += wpt) {
        const int sl = g.halves == 2 ? u >> 1 : u, half = u & 1;
        const uint8_t* cA = st + (ta * g.sbs + sl) * g.cb;
        const uint8_t* cB = st + (tb * g.sbs + sl) * g.cb;
        const int sbg = part * g.sbs + sl;
#pragma unroll
        for (int ps = 0; ps < P; ps++) {
            if (ps * NTK >= nc) break;
            const int nt = min(NTK, nc - ps * NTK);
            if (res_bytes > 0) {
                const uint8_t* tq[NTK];
#pragma unroll
                for (int q = 0; q < NTK; q++) tq[q] = res + h[8 + ps * NTK + min(q, nt - 1)] * cfg.xtab_bytes;
                if (g.halves == 1) stream_unit<FMT, NTK, true, true>(cA, cB, tq, nt, K, sbg, 0, lane, bm, y[ps]);
                else stream_unit<FMT, NTK, true, false>(cA, cB, tq, nt, K, sbg, half, lane, bm, y[ps]);
            } else {
                const uint8_t* tq[NTK];
#pragma unroll
                for (int q = 0; q < NTK; q++) tq[q] = p.xtab + (size_t)h[8 + ps * NTK + min(q, nt - 1)] * p.xtab_stride;
                if (g.halves == 1) stream_unit<FMT, NTK, false, true>(cA, cB, tq, nt, K, sbg, 0, lane, bm, y[ps]);
                else stream_unit<FMT, NTK, false, false>(cA, cB, tq, nt, K, sbg, half, lane, bm, y[ps]);
            }
        }
    }
}

// ------------------------------------------------------------ kernel
// Producer: the copies of one stage (lanes in parallel).  Gate/up (M = 2):
// the r16 gate tiles then the r16 up tiles; down (M = 1): 2*r16 consecutive
// 8-row tiles.  One copy per tile's K range, or one per matrix when the stage
// holds whole rows (the tiles are then consecutive in HBM).
template <int M>
__device__ __forceinline__ void stream_issue(const StreamSeg& g, const MatDev* md, int rg, int part, uint8_t* st,
                                             uint64_t* bar, int lane) {
    const int nsb = g.parts * g.sbs;
    const size_t run = (size_t)g.sbs * g.cb;
    if (g.parts == 1) {
        // whole rows: one copy per matrix
        constexpr int NM = M;
        for (int c = lane; c < NM; c += 32) {
            const MatDev mat = md[M == 2 ? c : 2];
            const int nt = M == 2 ? g.r16 : 2 * g.r16;           // 8-row tiles in the run
            const long long t0 = (long long)rg * nt;
            bulk_g2s(st + (size_t)c * nt * run, mat.base + t0 * nsb * g.cb, (uint32_t)(nt * run), bar);
        }
        return;
    }
    const int ntile = 2 * g.r16;
    for (int c = lane; c < ntile; c += 32) {
        int m, tile;
        if (M == 2) { m = c / g.r16; tile = rg * g.r16 + (c - m * g.r16); }
        else { m = 2; tile = rg * ntile + c; }
        const MatDev mat = md[m];
        bulk_g2s(st + (size_t)c * run, mat.base + ((long long)tile * nsb + (long long)part * g.sbs) * g.cb,
                 (uint32_t)run, bar);
    }
}

// Expert parallelism (down launches that store into the owners' mailboxes):
// a consumer warp that has finished all its work counts itself; the last of
// the grid's cw * gridDim.x consumer warps makes every row store of the grid
// visible system-wide and raises this rank's output flag at every owner.
__device__ __forceinline__ void stream_ep_done(const GemvParams& p, int cw, int lane) {
    __syncwarp();
    if (lane != 0) return;
    __threadfence_system();
    if (atomicAdd(p.ep_cnt, 1u) != (uint32_t)(cw * gridDim.x) - 1u) return;
    *p.ep_cnt = 0u;
    __threadfence_system();
    const uint32_t epoch = *p.ep_epoch;
    for (int q = 0; q < p.ep_G; q++) {
        uint32_t* f = reinterpret_cast<uint32_t*>(reinterpret_cast<char*>(p.ep_base[q]) + p.ep_flag) + p.ep_rank;
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(f), "r"(epoch) : "memory");
    }
}

// Registers: a sub-partition holds 16K; with 17 warps one holds 5, so a
// thread gets 96 registers, with 15 warps 128.
template <int FA, int FB, int M, int NTK>
__global__ void __launch_bounds__(32 * ((NTK == 1 ? kStreamMaxWarps : kStreamMaxWarps2) + 1), 1)
expert_stream_kernel(GemvParams p, StreamConfig cfg, int32_t* err) {
    constexpr int P = stream_passes(NTK), C = stream_chunk(NTK);
    extern __shared__ __align__(128) uint8_t ssm[];
    const int S = cfg.stages;
    uint64_t* full = reinterpret_cast<uint64_t*>(ssm);
    uint64_t* empty = full + kStreamMaxStages;
    uint64_t* tabbar = empty + kStreamMaxStages;
    int* ctl = reinterpret_cast<int*>(ssm + kStreamCtlOff);
    volatile int* abort_flag = ctl;
    int* hdr = reinterpret_cast<int*>(ssm + kStreamHdrOff);   // [stage][kStreamHdrInts]
    const int res_bytes = cfg.res_rows * cfg.xtab_bytes;
    const StreamRed R{ctl + 4, ctl + 8, reinterpret_cast<float*>(ssm + kStreamDataOff + res_bytes), cfg.red_bytes / 4};
    uint8_t* data = ssm + kStreamDataOff + res_bytes + kStreamRedSlots * cfg.red_bytes;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int CW = cfg.cw;
    const int K = p.cols;

    if (tid == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], CW);
        }
        mbar_init(tabbar, 1);
        *abort_flag = 0;
        for (int q = 0; q < kStreamRedSlots; q++) R.arr[q] = R.tick[q] = 0;
        fence_barrier_init();
    }
    __syncthreads();
    // the producer of a down launch may stream weights before the predecessor
    // (gate/up) has finished; everything else waits for it
    if (p.pdl == 1 || warp != CW) pdl_wait();
    pdl_trigger();
    const int n_active = *p.n_active;
    const int nA = p.mode == 2 ? 0 : n_active * cfg.seg[0].items_per_slot;
    const int nB = (p.mode == 1 || !p.has_shared) ? 0 : cfg.seg[1].items_per_slot;
    const int n_items = nA + nB;

    if (warp == CW) {
        // ---------------- producer: the lanes resolve the CTA's next 32 items
        // (expert, token run) at once; lane 0 waits for free stages and
        // writes the stage headers; the lanes issue the copies in parallel
        if (p.pdl == 2 && !p.xq_a) pdl_wait();   // tables written by the predecessor
        if (lane == 0 && res_bytes > 0 && !p.xq_a) {
            mbar_arrive_expect_tx(tabbar, (uint32_t)res_bytes);
            bulk_g2s(ssm + kStreamDataOff, p.xtab, (uint32_t)res_bytes, tabbar);
        }
        struct Item { int seg, slot, rg, e, off, n_tok, tok0, pad; };
        static_assert(sizeof(Item) == kStreamItemBytes, "item table entry");
        Item* items = reinterpret_cast<Item*>(ssm + kStreamItemOff);
        auto resolve = [&](int item, Item& in) {
            if (item < nA) {
                in.seg = 0;
                in.slot = item / cfg.seg[0].items_per_slot;
                in.rg = item - in.slot * cfg.seg[0].items_per_slot;
            } else {
                in.seg = 1;
                in.slot = n_active;
                in.rg = item - nA;
            }
            in.tok0 = -1;
            if (p.slot_info && in.seg == 0) {
                const int4 si = p.slot_info[in.slot];   // expert, first position, tokens, first token
                in.e = si.x; in.off = si.y; in.n_tok = si.z; in.tok0 = si.w;
            } else {
                in.e = p.active[in.slot];
                in.off = 0;
                in.n_tok = p.T_sh;
                if (in.seg == 0) { in.off = p.offsets[in.e]; in.n_tok = p.offsets[in.e + 1] - in.off; }
            }
        };
        bool ok = true;
        int k = 0;   // stages issued
        for (int idx = 0, item = blockIdx.x; ok; idx++, item += gridDim.x) {
            if (item >= n_items) {
                // end marker in the next stage
                const int s = k % S;
                const uint32_t ph = (uint32_t)(k / S) & 1u;
                if (k >= S) {
                    const bool w = lane == 0 ? mbar_wait_abort(&empty[s], ph ^ 1u, abort_flag) : true;
                    if (!__shfl_sync(0xffffffffu, (int)w, 0)) { ok = false; break; }
                }
                if (lane == 0) {
                    hdr[s * kStreamHdrInts] = n_items;
                    mbar_arrive(&full[s]);
                }
                break;
            }
            // every lane resolves one of the next 32 items: one round of global
            // loads per 32 items instead of one per item
            if (idx % kStreamItemBatch == 0) {
                const int it2 = item + lane * (int)gridDim.x;
                if (it2 < n_items) resolve(it2, items[lane]);
                __syncwarp();
            }
            const Item cur = items[idx % kStreamItemBatch];
            __syncwarp();
            const StreamSeg g = cur.seg ? cfg.seg[1] : cfg.seg[0];
            const MatDev* md = p.mats + (size_t)cur.e * 3;
            const int nchunk = (max(cur.n_tok, 1) + C - 1) / C;
            for (int c = 0; c < nchunk && ok; c++) {
                const int t0 = c * C, nc = max(0, min(C, cur.n_tok - t0));
                // table rows of the chunk's tokens
                int trow = 0;
                if (lane < nc) {
                    const int tk = t0 + lane;
                    if (cur.seg == 1) trow = p.xtab_shared_base + tk;
                    else if (p.routed_by_token) trow = (tk == 0 && cur.tok0 >= 0) ? cur.tok0 : p.pos_tok[cur.off + tk];
                    else trow = cur.off + tk;
                }
                for (int part = 0; part < g.parts; part++) {
                    const int s = k % S;
                    const uint32_t ph = (uint32_t)(k / S) & 1u;
                    if (k >= S) {
                        const bool w = lane == 0 ? mbar_wait_abort(&empty[s], ph ^ 1u, abort_flag) : true;
                        if (!__shfl_sync(0xffffffffu, (int)w, 0)) { ok = false; break; }
                    }
                    int* h = hdr + s * kStreamHdrInts;
                    if (lane < kStreamMaxChunk) h[8 + lane] = lane < nc ? trow : 0;
                    if (lane == 0) {
                        h[0] = item; h[1] = cur.slot; h[2] = cur.e; h[3] = cur.off; h[4] = nc;
                        h[5] = cur.seg; h[6] = part; h[7] = cur.rg | (t0 << 16);
                        mbar_arrive_expect_tx(&full[s], (uint32_t)g.stage_bytes);
                    }
                    __syncwarp();
                    uint8_t* st = data + (size_t)s * cfg.stage_bytes;
                    stream_issue<M>(g, md, cur.rg, part, st, &full[s], lane);
                    k++;
                }
            }
        }
        if (lane == 0) {
            if (!ok) {
                *abort_flag = 1;
                atomicOr(err, (int)ERR_TIMEOUT);
                // the stages this warp filled must land before the CTA exits
                for (int i = max(0, k - S); i < k; i++) mbar_wait(&full[i % S], (uint32_t)(i / S) & 1u);
            }
            if (res_bytes > 0 && !p.xq_a) mbar_wait(tabbar, 0u);
        }
        return;
    }

    // ---------------- consumers
    const int gid = lane >> 2;
    uint32_t bm[4];   // B column pair (2j, 2j+1) of group j: lanes gid = 2j, 2j+1 supply it
#pragma unroll
    for (int g4 = 0; g4 < 4; g4++) bm[g4] = (gid >> 1) == g4 ? 0xFFFFFFFFu : 0u;
    if (res_bytes > 0 && p.xq_a) {
        // quantise the resident tables here from the f32 rows (rows < xq_split
        // from xq_a, the rest from xq_b) while the first stages stream in; no
        // consumer leaves before this barrier
        const int quads = K / 128, total = cfg.res_rows * quads;
        for (int base = warp; base < total; base += 8 * CW) {
            float4 v[8];
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const int w = base + u * CW;
                if (w < total) {
                    const int r = w / quads, c = w - r * quads;
                    const float* src = r < p.xq_split ? p.xq_a + (size_t)r * K : p.xq_b + (size_t)(r - p.xq_split) * K;
                    v[u] = __ldcg(reinterpret_cast<const float4*>(src) + 32 * c + lane);
                }
            }
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const int w = base + u * CW;
                if (w < total) {
                    const int r = w / quads, c = w - r * quads;
                    xquant_quad(v[u], lane, c, K, ssm + kStreamDataOff + r * cfg.xtab_bytes);
                }
            }
        }
        named_barrier(1, CW * 32);
    } else if (res_bytes > 0 && !warp_wait(tabbar, 0u, abort_flag, err)) {
        return;
    }
    const uint8_t* res = ssm + kStreamDataOff;
    float y[P][NTK][2];
    int rseq = 0;   // reductions this warp has taken part in (the same for every warp)
    for (int k = 0;; k++) {
        const int s = k % S;
        const uint32_t ph = (uint32_t)(k / S) & 1u;
        if (!warp_wait(&full[s], ph, abort_flag, err)) return;
        const int* h = hdr + s * kStreamHdrInts;
        if (h[0] >= n_items) {
            if (M == 1 && p.ep_base) stream_ep_done(p, CW, lane);
            break;
        }
        const int seg = h[5], part = h[6];
        const StreamSeg& g = seg ? cfg.seg[1] : cfg.seg[0];
        if (part == 0) {
#pragma unroll
            for (int ps = 0; ps < P; ps++)
#pragma unroll
                for (int q = 0; q < NTK; q++) y[ps][q][0] = y[ps][q][1] = 0.f;
        }
        const uint8_t* st = data + (size_t)s * cfg.stage_bytes;
        if (seg == 0) stream_stage<FA, M, NTK>(p, cfg, g, h, st, res, warp, lane, bm, y);
        else stream_stage<FB, M, NTK>(p, cfg, g, h, st, res, warp, lane, bm, y);
        // what the reduction needs, before the stage (and its header) is released
        const int nc = h[4], slot = h[1], off = h[3], rg = h[7] & 0xFFFF, t0 = h[7] >> 16;
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);   // this warp is done with the stage
        if (part != g.parts - 1 || nc <= 0) continue;
        // reduce over the 4 lanes of a row, publish the warp's partials
        const int r = rseq++;
        const int sq = r % kStreamRedSlots, ticket = r / kStreamRedSlots;
        if (!warp_spin_eq(&R.tick[sq], ticket, abort_flag, err)) return;
        float* red = R.buf + (size_t)sq * R.floats;
#pragma unroll
        for (int ps = 0; ps < P; ps++)
#pragma unroll
            for (int q = 0; q < NTK; q++)
#pragma unroll
                for (int hh = 0; hh < 2; hh++) {
                    float v = y[ps][q][hh];
                    v += __shfl_xor_sync(0xffffffffu, v, 1);
                    v += __shfl_xor_sync(0xffffffffu, v, 2);
                    const int tq = ps * NTK + q;
                    if ((lane & 3) == 0 && tq < nc) red[(warp * cfg.red_tok + tq) * 16 + gid + 8 * hh] = v;
                }
        __threadfence_block();
        __syncwarp();
        // the last warp to publish adds the partials (fixed order) and frees the slot
        int last = 0;
        if (lane == 0) last = atomicAdd(&R.arr[sq], 1) == CW - 1;
        if (__shfl_sync(0xffffffffu, last, 0)) {
            __threadfence_block();
            stream_reduce<M, NTK>(p, cfg, StreamJob{r, seg, rg, off, t0, nc, slot >= n_active ? 1 : 0}, R, lane);
        }
    }
}

}  // namespace qrm
