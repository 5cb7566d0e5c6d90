// qrmoe.cu -- the C ABI of libqrmoe.so (include/qrmoe.h): layer state in
// HBM, uploads, the forward launch sequence and the matrix operator API.
//
// Forward launch sequence on the layer's stream (all device-resident):
//   route      RMSNorm + router logits, bit-exact emulation (route.cuh)
//   topk       softmax / sigmoid top-k and combine weights (route.cuh)
//   dispatch   stable counting sort -> perm, offsets, active expert list
//   gate/up    fused dequant GEMV + SwiGLU over (expert, row tile) items
//   down       fused dequant GEMV
//   combine    weighted sum in slot order (+ residual, + shared expert)
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <map>
#include <mutex>
#include <tuple>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <ctime>
#include <string>
#include <utility>
#include <vector>

#include "../../include/qrmoe.h"
#include <nccl.h>

#include "combine.cuh"
#include "ep.cuh"
#include "common.cuh"
#include "gemv.cuh"
#include "gemv_tma.cuh"
#include "gemv_imma.cuh"
#include "gemv_stream.cuh"
#include "layout.cuh"
#include "route.cuh"
#include "umma_host.h"

extern "C" int qrm_synth_quantize_impl(int fmt, const float* src, long long n, void* dst, cudaStream_t s);
extern "C" int qrm_synth_gaussian_impl(float* dst, long long n, uint64_t seed, float sigma, cudaStream_t s);

namespace {

thread_local std::string g_err;

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_err = buf;
    return code;
}

#define QRM_NCCL(expr)                                                                          \
    do {                                                                                        \
        ncclResult_t r_ = (expr);                                                               \
        if (r_ != ncclSuccess) return fail(QRM_E_NCCL, "%s: %s", #expr, ncclGetErrorString(r_)); \
    } while (0)
#define QRM_CUDA(expr)                                                                          \
    do {                                                                                        \
        cudaError_t e_ = (expr);                                                                \
        if (e_ != cudaSuccess) return fail(QRM_E_CUDA, "%s: %s", #expr, cudaGetErrorString(e_)); \
    } while (0)

int64_t tensor_bytes(int fmt, int64_t rows, int64_t cols) {
    int bs, bb;
    if (!qrm::block_spec(fmt, &bs, &bb)) return -1;
    if (cols % bs != 0) return -1;
    return rows * (cols / bs) * bb;
}

const char* which_name(int which) { return which == 0 ? "w_gate" : which == 1 ? "w_up" : "w_down"; }

// Template dispatch of the expert GEMV kernel.
template <int FMT, int M, int R>
cudaError_t launch_gemv_nt(int nt, const qrm::GemvParams& p, int grid, int block, cudaStream_t s) {
    switch (nt) {
        case 1: qrm::expert_gemv_kernel<FMT, M, R, 1><<<grid, block, 0, s>>>(p); break;
        case 2: qrm::expert_gemv_kernel<FMT, M, R, 2><<<grid, block, 0, s>>>(p); break;
        default: qrm::expert_gemv_kernel<FMT, M, R, 4><<<grid, block, 0, s>>>(p); break;
    }
    return cudaGetLastError();
}

template <int FMT, int M, int R>
int gemv_occupancy(int nt, int block) {
    int nb = 0;
    switch (nt) {
        case 1: cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, qrm::expert_gemv_kernel<FMT, M, R, 1>, block, 0); break;
        case 2: cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, qrm::expert_gemv_kernel<FMT, M, R, 2>, block, 0); break;
        default: cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, qrm::expert_gemv_kernel<FMT, M, R, 4>, block, 0); break;
    }
    return std::max(nb, 1);
}

constexpr int kRGateUp = 4;   // rows per gate/up item (x2 matrices)
constexpr int kRDown = 8;     // rows per down item

// Router logits tiles (route.cuh): every instantiation gets its shared memory
// limit once; the launch takes the largest tile whose grid covers the SMs.
static bool lm_tiles_setup() {
    bool ok = true;
#define QRM_LM_SETUP(TT, TE, NTG, NEG, KC, NS)                                                           \
    ok = ok && cudaFuncSetAttribute(qrm::logits_lm_kernel<TT, TE, NTG, NEG, KC, NS>,                     \
                                    cudaFuncAttributeMaxDynamicSharedMemorySize,                         \
                                    (int)qrm::LMTile<TT, TE, NTG, NEG, KC, NS>::smem()) == cudaSuccess;
    QRM_LM_TILES(QRM_LM_SETUP)
#undef QRM_LM_SETUP
    return ok;
}

static void launch_logits_lm(const float* xn, const float* router_lm, const float* offset, float* logits, int T, int d,
                             int E, int sm_count, cudaStream_t s) {
    bool done = false;
#define QRM_LM_COUNT(TT, TE, NTG, NEG, KC, NS) +1
    int left = 0 QRM_LM_TILES(QRM_LM_COUNT);   // the last tile runs whatever its grid
#undef QRM_LM_COUNT
#define QRM_LM_LAUNCH(TT, TE, NTG, NEG, KC, NS)                                                          \
    if (!done) {                                                                                          \
        using Tl = qrm::LMTile<TT, TE, NTG, NEG, KC, NS>;                                                 \
        const dim3 grid((T + Tl::kT - 1) / Tl::kT, (E + Tl::kE - 1) / Tl::kE);                          \
        if (--left == 0 || (long long)grid.x * grid.y >= sm_count) {                                      \
            qrm::logits_lm_kernel<TT, TE, NTG, NEG, KC, NS><<<grid, Tl::kThreads, Tl::smem(), s>>>(       \
                xn, router_lm, offset, logits, T, d, E);                                                  \
            done = true;                                                                                  \
        }                                                                                                 \
    }
    QRM_LM_TILES(QRM_LM_LAUNCH)
#undef QRM_LM_LAUNCH
}

// Bulk-copy staged kernel: G consumer groups, NT tokens per pass.
template <int FMT, int M, int R, int NT, int G>
int launch_tma_g(const qrm::GemvParams& p, const qrm::TmaConfig& cfg, int cwg, int sm_count, int32_t* err,
                 cudaStream_t s) {
    auto fn = qrm::expert_gemv_tma_kernel<FMT, M, R, NT, G>;
    const size_t smem = qrm::tma_smem_bytes(cfg);
    static bool attr_set = false;  // one per instantiation
    if (!attr_set) {
        if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) != cudaSuccess)
            return fail(QRM_E_CUDA, "expert kernel attribute");
        attr_set = true;
    }
    fn<<<sm_count, (G * cwg + 1) * 32, smem, s>>>(p, cfg, err);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? QRM_OK : fail(QRM_E_CUDA, "expert kernel launch: %s", cudaGetErrorString(e));
}

// Pick the tile height R, consumer groups G and tokens per pass NT:
// gate/up R = 8 (16 matrix rows per item); down R = 32 when the row is short
// enough for 4+ consumer groups, else 8.  NT keeps pairs*NT <= 32.
template <int FMT, int M, int R>
int launch_tma_r(int nt, const qrm::GemvParams& p, int sm_count, int32_t* err, cudaStream_t s, bool* used) {
    qrm::TmaConfig cfg;
    *used = false;
    if (p.rows % R) return QRM_OK;
    qrm::GemvParams q = p;
    q.tiles = p.rows / R;
    if (!qrm::tma_plan<FMT>(M, R, p.cols, 227 * 1024, &cfg)) return QRM_OK;
    const int cwg = (p.cols / 32 + 31) / 32;
    int G = 16;
    while (G > 1 && (G * cwg > 16 || (M * R) % G)) G >>= 1;
    constexpr int kPairsMax = M * R;
    const int pairs = kPairsMax / G;
    if (M == 1 && R == 32 && G < 4) return QRM_OK;   // caller falls back to R = 8
    *used = true;
    const bool one = nt <= 1 || pairs > 8;
#define QRM_TMA_G(GG)                                                                             \
    case GG:                                                                                      \
        if constexpr ((M * R) % GG == 0 && (M * R) / GG <= 32) {                                  \
            if (one || (M * R) / GG > 8) return launch_tma_g<FMT, M, R, 1, GG>(q, cfg, cwg, sm_count, err, s); \
            if constexpr ((M * R) / GG <= 8) return launch_tma_g<FMT, M, R, 4, GG>(q, cfg, cwg, sm_count, err, s); \
        }                                                                                         \
        break;
    switch (G) {
        QRM_TMA_G(16)
        QRM_TMA_G(8)
        QRM_TMA_G(4)
        QRM_TMA_G(2)
        QRM_TMA_G(1)
        default: break;
    }
#undef QRM_TMA_G
    *used = false;
    return QRM_OK;
}

template <int FMT, int M>
int launch_tma(int nt, const qrm::GemvParams& p, int sm_count, int32_t* err, cudaStream_t s, bool* used) {
    if (M == 1) {
        int rc = launch_tma_r<FMT, 1, 32>(nt, p, sm_count, err, s, used);
        if (rc || *used) return rc;
    }
    return launch_tma_r<FMT, M, 8>(nt, p, sm_count, err, s, used);
}

// Integer tensor-core kernel (Q4_K, Q8_0, Q4_0 with 256-multiple rows);
// needs the activation tables of p.xtab (written by xquant_kernel).

// Expert-parallel forwards are captured into CUDA graphs with their NCCL
// calls (QRM_EP_GRAPH=0 launches them directly).
bool ep_graphs_enabled() {
    static int v = -1;
    if (v < 0) {
        const char* e = getenv("QRM_EP_GRAPH");
        v = (e && e[0] == '0') ? 0 : 1;
    }
    return v == 1;
}

// Programmatic dependent launches between the forward's kernels, as a mask:
// 1 gate/up, 2 down, 4 combine.  On B200 the expert launches ran slower as
// dependents (measured 7570 -> 6966 / 7234 tokens/s at C5, T = 1), the
// combine slightly faster, so only the combine is (QRM_PDL overrides the mask
// for tuning runs).
int pdl_default() {
    const char* e = getenv("QRM_PDL");
    return e ? atoi(e) : 4;
}

// Launches kern, as a programmatic dependent of the previous launch on s when
// pdl is set (the kernel then calls pdl_wait before it reads that launch's
// outputs).
template <typename... KArgs, typename... Args>
cudaError_t launch_k(bool pdl, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                     Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// The streaming integer kernel's launch shape for one matrix launch.
struct StreamSel {
    int ntk = 1;
    qrm::StreamConfig cfg{};
};

bool imma_format(int fmt) { return fmt == qrm::Q4_K || fmt == qrm::Q8_0 || fmt == qrm::Q4_0; }

// true when a matrix of this shape is stored in the tiled layout and taken by
// the streaming integer kernel (tables wanted); gate/up pairs 8-row tiles of
// the two matrices, down takes 16 rows per MMA tile
bool imma_usable(int fmt, int rows, int cols, bool gateup) {
    if (!imma_format(fmt) || cols % 256) return false;
    return rows % (gateup ? 8 : 16) == 0;
}

// Shapes the tcgen05 grouped path takes: gate/up rows in blocks of 64, down
// rows in blocks of 128, both K ranges whole super-blocks.
bool umma_shapes(int d, int f) { return f % 64 == 0 && d % 128 == 0 && d % 256 == 0 && f % 256 == 0; }

// true when an expert matrix of a layer with d_model d and expert_ffn f is
// stored in the tiled layout: the integer streaming kernel's formats as
// before, Q6_K and TRI when the grouped path takes the layer's shapes (it is
// then their kernel at every batch size)
bool layer_tiled(int fmt, int d, int f, bool gateup) {
    const int rows = gateup ? f : d, cols = gateup ? d : f;
    if (imma_format(fmt)) return imma_usable(fmt, rows, cols, gateup);
    return (fmt == qrm::Q6_K || fmt == qrm::TRI) && umma_shapes(d, f);
}
bool umma_only_format(int fmt) { return fmt == qrm::Q6_K || fmt == qrm::TRI; }

// Plans a launch whose routed items use format fa and shared items format fb
// (-1: none); false when no plan fits (the caller reports it).
// Largest launch batch that takes the one-token-per-pass kernel: an expert
// slot with more tokens then streams its weights once per token, which at two
// tokens (single-GPU T = 2, or expert-parallel decode over two ranks) is rare
// and cheaper than the two-token kernel's geometry (14 warps, more registers):
// measured C5 T = 2 181 -> 164 us, two-GPU decode 166 -> 151 us.
// QRM_STREAM_NTK1_MAX overrides it for tuning runs.
int stream_ntk1_max() {
    static int v = -1;
    if (v < 0) {
        const char* e = getenv("QRM_STREAM_NTK1_MAX");
        v = e ? std::max(1, atoi(e)) : 2;
    }
    return v;
}

bool stream_select(int fa, int fb, bool gateup, int T, const qrm::GemvParams& p, int sm_count, StreamSel* sel) {
    if (!p.xtab) return false;
    if (fa >= 0 && !imma_usable(fa, p.rows, p.cols, gateup)) return false;
    if (fb >= 0 && !imma_usable(fb, p.rows, p.cols, gateup)) return false;
    sel->ntk = T <= stream_ntk1_max() ? 1 : 2;
    const int fmts[2] = {fa, fb};
    // larger down items only while the launch keeps two items per SM (the
    // routed slots are at most min(E, T*k))
    const int M = gateup ? 2 : 1;
    int max_r16 = qrm::stream_max_r16(M);
    if (max_r16 > qrm::kStreamMaxR16) {
        const long long slots = (fa >= 0 ? std::min<long long>(p.E, (long long)T * p.k) : 0) + (fb >= 0 ? 1 : 0);
        if (slots * (p.rows / (16 * max_r16)) < 2LL * sm_count) max_r16 = qrm::kStreamMaxR16;
    }
    return qrm::stream_plan(fmts, M, p.rows, p.cols, sel->ntk, p.xtab_rows, T, 227 * 1024, max_r16, &sel->cfg);
}

// segment formats of a launch of mode p.mode whose matrices are all format fmt
void imma_seg_fmts(int fmt, const qrm::GemvParams& p, int* fa, int* fb) {
    *fa = p.mode == 2 ? -1 : fmt;
    *fb = (p.mode == 1 || !p.has_shared) ? -1 : fmt;
}

template <int FA, int FB, int M, int NTK>
int launch_stream_t(const qrm::GemvParams& p, const StreamSel& sel, int sm_count, int32_t* err, cudaStream_t s) {
    auto fn = qrm::expert_stream_kernel<FA, FB, M, NTK>;
    static bool attr_set = false;
    if (!attr_set) {
        if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) != cudaSuccess)
            return fail(QRM_E_CUDA, "expert kernel attribute");
        attr_set = true;
    }
    cudaError_t e = launch_k(p.pdl != 0, fn, dim3(sm_count), dim3((sel.cfg.cw + 1) * 32),
                             qrm::stream_smem_bytes(sel.cfg), s, p, sel.cfg, err);
    if (e == cudaSuccess) e = cudaGetLastError();
    return e == cudaSuccess ? QRM_OK : fail(QRM_E_CUDA, "expert kernel launch: %s", cudaGetErrorString(e));
}

// the streaming kernel for segment formats (FA, FB); the matrices are tiled,
// so no other kernel can take the launch
template <int FA, int FB, int M>
int launch_stream(int fa, int fb, int T, const qrm::GemvParams& p, int sm_count, int32_t* err, cudaStream_t s) {
    StreamSel sel;
    if (!stream_select(fa, fb, M == 2, T, p, sm_count, &sel))
        return fail(QRM_E_STATE, "internal: no stage plan for the %d x %d expert matrices", p.rows, p.cols);
    // in-kernel tables only with a resident plan (the caller checked)
    if (p.xq_a && sel.cfg.res_rows == 0) return fail(QRM_E_STATE, "internal: activation tables were not built");
    return sel.ntk == 1 ? launch_stream_t<FA, FB, M, 1>(p, sel, sm_count, err, s)
                        : launch_stream_t<FA, FB, M, 2>(p, sel, sm_count, err, s);
}

// routed items in Q4_K and a Q8_0 shared expert in one launch (mode 0)
bool imma_pair_supported(int fa, int fb) { return fa == qrm::Q4_K && fb == qrm::Q8_0; }
int launch_stream_pair(bool gateup, int T, const qrm::GemvParams& p, int sm_count, int32_t* err, cudaStream_t s) {
    return gateup ? launch_stream<qrm::Q4_K, qrm::Q8_0, 2>(qrm::Q4_K, qrm::Q8_0, T, p, sm_count, err, s)
                  : launch_stream<qrm::Q4_K, qrm::Q8_0, 1>(qrm::Q4_K, qrm::Q8_0, T, p, sm_count, err, s);
}

// rows < split from src, the rest from src_b (row r - split)
int launch_xquant(const float* src, int K, int rows, uint8_t* tab, cudaStream_t s, const float* src_b = nullptr,
                  int split = -1) {
    if (rows <= 0) return QRM_OK;
    if (split < 0) split = rows;
    long long warps = (long long)rows * (K / 32);
    int grid = (int)std::min<long long>((warps + 7) / 8, 148 * 16);
    qrm::xquant_kernel<<<grid, 256, 0, s>>>(src, src_b, split, K, rows, tab, qrm::xtab_stride(K));
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? QRM_OK : fail(QRM_E_CUDA, "xquant launch: %s", cudaGetErrorString(e));
}

// gate/up (M=2) or down (M=1) for one format: the integer tensor-core kernel
// for Q4_K / Q8_0 / Q4_0, else the bulk-copy staged kernel
// when the tile fields are 16-byte multiples, else the register kernel.
int launch_gemv(int fmt, bool gateup, int nt, const qrm::GemvParams& p, int sm_count, int32_t* err, cudaStream_t s) {
    const int U = p.cols / 32;
    const int block = (U + 31) / 32 * 32;
    int occ = 1;
    cudaError_t e = cudaSuccess;
    bool used = false;
    int rc = QRM_OK;
#define QRM_GEMV_CASE(F)                                                                        \
    case F:                                                                                     \
        if (imma_usable(F, p.rows, p.cols, gateup)) {                                           \
            constexpr int FI = (F == qrm::Q4_K || F == qrm::Q8_0 || F == qrm::Q4_0) ? F : qrm::Q4_K;  \
            int fa, fb;                                                                         \
            imma_seg_fmts(F, p, &fa, &fb);                                                      \
            return gateup ? launch_stream<FI, FI, 2>(fa, fb, p.T, p, sm_count, err, s)           \
                          : launch_stream<FI, FI, 1>(fa, fb, p.T, p, sm_count, err, s);          \
        }                                                                                       \
        if (gateup) {                                                                           \
            rc = launch_tma<F, 2>(nt, p, sm_count, err, s, &used);                    \
            if (rc || used) return rc;                                                          \
            occ = gemv_occupancy<F, 2, kRGateUp>(nt, block);                                    \
            e = launch_gemv_nt<F, 2, kRGateUp>(nt, p, sm_count * occ, block, s);                \
        } else {                                                                                \
            rc = launch_tma<F, 1>(nt, p, sm_count, err, s, &used);                      \
            if (rc || used) return rc;                                                          \
            occ = gemv_occupancy<F, 1, kRDown>(nt, block);                                      \
            e = launch_gemv_nt<F, 1, kRDown>(nt, p, sm_count * occ, block, s);                  \
        }                                                                                       \
        break;
    // formats stored as in .qw: the register kernel
#define QRM_GEMV_RAW(F)                                                                         \
    case F:                                                                                     \
        if (gateup) {                                                                           \
            occ = gemv_occupancy<F, 2, kRGateUp>(nt, block);                                    \
            e = launch_gemv_nt<F, 2, kRGateUp>(nt, p, sm_count * occ, block, s);                \
        } else {                                                                                \
            occ = gemv_occupancy<F, 1, kRDown>(nt, block);                                      \
            e = launch_gemv_nt<F, 1, kRDown>(nt, p, sm_count * occ, block, s);                  \
        }                                                                                       \
        break;
    switch (fmt) {
        QRM_GEMV_CASE(qrm::Q4_K)
        QRM_GEMV_CASE(qrm::Q4_0)
        QRM_GEMV_CASE(qrm::Q8_0)
        QRM_GEMV_CASE(qrm::Q6_K)
        QRM_GEMV_CASE(qrm::TRI)
        QRM_GEMV_RAW(qrm::Q2_K)
        QRM_GEMV_RAW(qrm::Q3_K)
        QRM_GEMV_RAW(qrm::Q5_K)
        QRM_GEMV_RAW(qrm::I8_BLK)
        QRM_GEMV_RAW(qrm::B1)
        QRM_GEMV_RAW(qrm::B1X)
        QRM_GEMV_RAW(qrm::T1E)
        QRM_GEMV_RAW(qrm::T1E_LO)
        default: return fail(QRM_E_FORMAT, "format %d has no expert kernel", fmt);
    }
#undef QRM_GEMV_CASE
#undef QRM_GEMV_RAW
    if (e != cudaSuccess) return fail(QRM_E_CUDA, "expert kernel launch: %s", cudaGetErrorString(e));
    return QRM_OK;
}

int pick_nt(int T) { return T <= 1 ? 1 : (T <= 8 ? 2 : 4); }

}  // namespace

// ---------------------------------------------------------------- layer

struct qrm_layer {
    qrm_layer_desc desc{};
    int k = 0;
    int first_expert = 0, n_local = 0;  // routed experts held by this layer
    // expert parallelism: rank of world, one NCCL communicator per layer
    int world = 1, rank = 0;
    ncclComm_t comm = nullptr;
    float* rec_own = nullptr;     // [T][d + 2k] this rank's (xn, top-k idx, top-k w) records
    float* rec_all = nullptr;     // [world*T][d + 2k] gathered records
    float* xn_all = nullptr;      // [world*T][d]
    int32_t* idx_all = nullptr;   // [world*T][k]
    float* ysend = nullptr;       // [world][T*k][d] output rows per owner (NCCL)
    float* yrecv = nullptr;       // rows of this rank's tokens: [T*k][d] in the mailbox (peer memory)
                                  // or [world][T*k][d] per holder (yrecv_nccl)
    float* yrecv_nccl = nullptr;
    // xn_all, idx_all (and yrecv) live in this rank's mailbox; in peer-memory
    // mode every rank maps every other rank's mailbox and writes into it
    char* mbox = nullptr;
    qrm::EpMailbox mb{};
    bool p2p = false;
    std::vector<void*> peer_open;             // mapped peer mailboxes
    unsigned long long* peer_base = nullptr;  // device [world]: mailbox of each rank
    uint32_t* ep_state = nullptr;             // device: epoch, block counters [2][world]
    char* xch = nullptr;                      // device [world][128]: set-up exchange, barrier
    bool shared_enabled = false;        // GLM layer with n_shared > 0
    int sm_count = 0;
    cudaStream_t stream = nullptr;
    // qrm_forward's pinned host staging (small batches, allocated on first use):
    // [cap rows][d] inputs | [cap rows][d] outputs | [cap rows][k] indices |
    // [cap rows][k] weights | error flags
    char* host_stage = nullptr;
    int host_stage_rows = 0;
    // device views of the staging's top-k and error flags while a staged
    // forward is captured (the combine copies them there); null otherwise
    int32_t* stage_idx = nullptr;
    float* stage_w = nullptr;
    int32_t* stage_err = nullptr;
    // weights
    uint8_t* slab = nullptr;
    size_t slab_bytes = 0;
    bool slab_owned = true;       // false: a slot of a qrm_stack (layer weights streamed into it)
    uint8_t* image = nullptr;     // streamed layer: pinned host copy of its slab in device layout
    std::vector<qrm::MatDev> mats;      // (E+1)*3
    std::vector<size_t> mat_bytes;
    qrm::MatDev* mats_dev = nullptr;
    std::vector<uint8_t> uploaded;      // (E+1)*3
    float* norm_w = nullptr;
    float* router = nullptr;
    float* router_lm = nullptr;   // lane-major copy of the router rows (fused router)
    float* router_bias = nullptr;
    float* offset = nullptr;
    bool has_norm = false, has_router = false, has_bias = false, has_offset = false;
    // work buffers
    int cap_T = 0;
    float *x = nullptr, *xn = nullptr, *logits = nullptr, *topk_w = nullptr;
    float *h = nullptr, *hs = nullptr, *y = nullptr, *ys = nullptr, *out = nullptr;
    int32_t *topk_idx = nullptr, *perm = nullptr, *inv_perm = nullptr, *offsets = nullptr, *active = nullptr;
    int32_t* pos_tok = nullptr;
    int4* slot_info = nullptr;    // per active slot: expert, first position, tokens, first token
    qrm::Schedule* sched = nullptr;
    uint8_t* staging = nullptr;
    size_t staging_bytes = 0;
    uint8_t* xtab_gu = nullptr;   // activation tables of the gate/up inputs [T]
    uint8_t* xtab_dn = nullptr;   // of the down inputs [T*k routed | T shared]
    // tcgen05 grouped path for large per-expert groups (umma.cu)
    bool umma_ok = false;         // formats and shapes allow it; buffers allocated
    int umma_mode = -1;           // -1 by group size, 0 never, 1 always (QRM_UMMA)
    bool umma_forced_gu = false;  // a gate/up format has no other kernel in the tiled layout (Q6_K, TRI)
    bool umma_forced_dn = false;  // same for down
    // average routed tokens per expert from which it is used (QRM_UMMA_MIN_TPE),
    // or shared-expert tokens: measured crossovers against the decode kernels
    // on B200 (configs 1-5: from 4 tokens per expert, or 64 shared tokens)
    int umma_min_tpe = 4;
    int umma_min_shared = 64;

    __half* act16 = nullptr;      // [Tx*k + Tx][d] f16 gate/up inputs in dispatch order
    __half* h16 = nullptr;        // [Tx*k + Tx][f] f16 down inputs
    qrm::UmmaItem* umma_items = nullptr;   // [2][cap]: gate/up items, down items
    int32_t* umma_count = nullptr;         // [2]
    long long umma_cap = 0;
    CUtensorMap act_map{}, h_map{};
    int last_T = 0;
    int last_launches = 0;        // kernel launches of the last forward
    const float* last_xn = nullptr;
    // per-stage timing
    bool profiling = false;
    int pdl = pdl_default();      // programmatic dependent launches in the forward graph (mask)
    bool profiled_last = false;
    cudaEvent_t ev[QRM_STAGE_COUNT + 1] = {};
    bool last_shared = false;
    // CUDA graphs of the forward, keyed by buffers, T, flags and profiling
    // one instantiated graph per (T, flags, profiling); a call with other buffers
    // re-captures and updates it in place (cudaGraphExecUpdate)
    using GraphKey = std::tuple<int, int, int>;
    struct Graph {
        cudaGraphExec_t exec = nullptr;
        int launches = 0;                // kernel launches in it
        const void* ptrs[4] = {};        // x, out, top-k idx, top-k w it was captured with
    };
    std::map<GraphKey, Graph> graphs;
};

static void clear_graphs(qrm_layer* L) {
    for (auto& kv : L->graphs) cudaGraphExecDestroy(kv.second.exec);
    L->graphs.clear();
}

// All ranks of an expert-parallel layer meet here (qrm_destroy is collective).
// Bounded: false when a rank did not arrive within ~10 s.
static bool ep_barrier(qrm_layer* L) {
    if (ncclAllReduce(L->xch, L->xch, 1, ncclInt32, ncclSum, L->comm, L->stream) != ncclSuccess) return false;
    for (int i = 0; i < 10000; i++) {
        cudaError_t e = cudaStreamQuery(L->stream);
        if (e == cudaSuccess) return true;
        if (e != cudaErrorNotReady) return false;
        struct timespec ts{0, 1000000};
        nanosleep(&ts, nullptr);
    }
    return false;
}

// Waits up to `ms` milliseconds for the stream's work to finish.
static bool drain_stream(cudaStream_t s, int ms) {
    for (int i = 0; i < ms; i++) {
        cudaError_t e = cudaStreamQuery(s);
        if (e == cudaSuccess) return true;
        if (e != cudaErrorNotReady) return false;
        struct timespec ts{0, 1000000};
        nanosleep(&ts, nullptr);
    }
    return false;
}

static void free_layer(qrm_layer* L) {
    if (!L) return;
    cudaSetDevice(L->desc.device);
    bool met = true;
    if (L->stream) {
        // an expert-parallel forward whose collective waits for a rank that
        // left never ends by itself: bounded
        if (L->world > 1) met = drain_stream(L->stream, 10000);
        else cudaStreamSynchronize(L->stream);
    }
    // every rank meets here before its mailbox goes away (no peer writes into
    // it afterwards); bounded, false when a rank did not arrive
    if (met && L->comm) met = ep_barrier(L);
    if (!met && L->comm) {
        // abort first: it ends this communicator's kernels still in flight, so
        // the device-synchronising calls below (stream sync, cudaFree) cannot
        // wait behind a collective that never completes
        ncclCommAbort(L->comm);
        L->comm = nullptr;
    }
    if (L->p2p) {
        for (void* p : L->peer_open) cudaIpcCloseMemHandle(p);
        L->peer_open.clear();
    }
    // a peer that may still write into it keeps the mailbox (leaked, not freed)
    if (L->mbox && met) cudaFree(L->mbox);
    if (!L->slab_owned) L->slab = nullptr;   // the stack's slot
    L->xn_all = nullptr;
    L->idx_all = nullptr;
    L->yrecv = nullptr;
    void* ptrs[] = {L->slab, L->mats_dev, L->norm_w, L->router, L->router_lm, L->router_bias, L->offset, L->x, L->xn,
                    L->logits, L->topk_w, L->h, L->hs, L->y, L->ys, L->out, L->topk_idx, L->perm,
                    L->inv_perm, L->offsets, L->active, L->sched, L->staging, L->xtab_gu, L->xtab_dn,
                    L->pos_tok, L->slot_info, L->act16, L->h16, L->umma_items, L->umma_count,
                    L->rec_own, L->rec_all, L->ysend, L->yrecv_nccl, L->peer_base, L->ep_state, L->xch};
    for (void* p : ptrs)
        if (p) cudaFree(p);
    if (L->host_stage) cudaFreeHost(L->host_stage);
    clear_graphs(L);
    for (cudaEvent_t e : L->ev)
        if (e) cudaEventDestroy(e);
    if (L->stream) cudaStreamDestroy(L->stream);
    if (L->comm) ncclCommDestroy(L->comm);   // every rank met: nothing of it is in flight
    delete L;
}

static int check_desc(const qrm_layer_desc* d) {
    if (!d) return fail(QRM_E_INVALID, "desc is NULL");
    if (d->d_model <= 0 || d->expert_ffn <= 0 || d->n_experts <= 0 || d->n_active <= 0)
        return fail(QRM_E_INVALID, "d_model, expert_ffn, n_experts and n_active must be positive");
    if (d->n_experts > qrm::kMaxE) return fail(QRM_E_CAPACITY, "n_experts %d > %d", d->n_experts, qrm::kMaxE);
    if (std::min(d->n_active, 8) > d->n_experts) return fail(QRM_E_INVALID, "top-k exceeds n_experts");
    if (d->d_model % 32 || d->expert_ffn % 32) return fail(QRM_E_INVALID, "d_model and expert_ffn must be multiples of 32");
    if (d->d_model / 32 > qrm::kGemvMaxThreads || d->expert_ffn / 32 > qrm::kGemvMaxThreads)
        return fail(QRM_E_CAPACITY, "rows longer than %d columns are not supported", 32 * qrm::kGemvMaxThreads);
    if (d->max_tokens <= 0) return fail(QRM_E_INVALID, "max_tokens must be positive");
    const int fm[6] = {d->fmt_gate, d->fmt_up, d->fmt_down, d->fmt_sh_gate, d->fmt_sh_up, d->fmt_sh_down};
    const bool shared = d->moe_sigmoid && d->n_shared > 0;
    for (int i = 0; i < (shared ? 6 : 3); i++) {
        if (!qrm::is_expert_fmt(fm[i])) return fail(QRM_E_FORMAT, "format %d is not an expert format", fm[i]);
        int bs, bb;
        qrm::block_spec(fm[i], &bs, &bb);
        int cols = (i % 3 == 2) ? d->expert_ffn : d->d_model;
        if (cols % bs) return fail(QRM_E_INVALID, "%d columns are not a multiple of the %d-weight block", cols, bs);
    }
    if (d->fmt_gate != d->fmt_up || (shared && d->fmt_sh_gate != d->fmt_sh_up))
        return fail(QRM_E_FORMAT, "gate and up must share a format");
    return QRM_OK;
}

static int alloc_work(qrm_layer* L, int T) {
    const int d = L->desc.d_model, E = L->desc.n_experts, f = L->desc.expert_ffn, k = L->k;
    const size_t Tk = (size_t)T * k;
    QRM_CUDA(cudaMalloc(&L->x, sizeof(float) * T * d));
    QRM_CUDA(cudaMalloc(&L->xn, sizeof(float) * T * d));
    QRM_CUDA(cudaMalloc(&L->out, sizeof(float) * T * d));
    QRM_CUDA(cudaMalloc(&L->logits, sizeof(float) * T * E));
    QRM_CUDA(cudaMalloc(&L->topk_w, sizeof(float) * Tk));
    QRM_CUDA(cudaMalloc(&L->topk_idx, sizeof(int32_t) * Tk));
    QRM_CUDA(cudaMalloc(&L->perm, sizeof(int32_t) * Tk));
    QRM_CUDA(cudaMalloc(&L->inv_perm, sizeof(int32_t) * Tk));
    QRM_CUDA(cudaMalloc(&L->pos_tok, sizeof(int32_t) * Tk));
    QRM_CUDA(cudaMalloc(&L->slot_info, sizeof(int4) * (E + 1)));
    QRM_CUDA(cudaMalloc(&L->offsets, sizeof(int32_t) * (E + 1)));
    QRM_CUDA(cudaMalloc(&L->active, sizeof(int32_t) * (E + 1)));
    QRM_CUDA(cudaMalloc(&L->sched, sizeof(qrm::Schedule)));
    QRM_CUDA(cudaMemset(L->sched, 0, sizeof(qrm::Schedule)));
    QRM_CUDA(cudaMalloc(&L->h, sizeof(float) * Tk * f));
    QRM_CUDA(cudaMalloc(&L->y, sizeof(float) * Tk * d));
    if (L->shared_enabled) {
        QRM_CUDA(cudaMalloc(&L->hs, sizeof(float) * T * f));
        QRM_CUDA(cudaMalloc(&L->ys, sizeof(float) * T * d));
    }
    QRM_CUDA(cudaMalloc(&L->xtab_gu, (size_t)qrm::xtab_stride(d) * T));
    QRM_CUDA(cudaMalloc(&L->xtab_dn, (size_t)qrm::xtab_stride(f) * (Tk + T)));
    L->cap_T = T;
    return QRM_OK;
}

extern "C" int qrm_version(void) { return QRM_ABI_VERSION; }
// the error text of this thread's last failing call, for the other
// translation units of the library (not exported)
extern "C" __attribute__((visibility("hidden"))) int qrm_set_error(int code, const char* msg) {
    return fail(code, "%s", msg);
}
extern "C" const char* qrm_last_error(void) { return g_err.c_str(); }

static int create_layer(const qrm_layer_desc* desc, int rank, int world, const void* nccl_id, qrm_layer** out,
                        uint8_t* ext_slab = nullptr);

extern "C" int qrm_create(const qrm_layer_desc* desc, qrm_layer** out) {
    return create_layer(desc, 0, 1, nullptr, out);
}

extern "C" int qrm_nccl_unique_id(void* id_out) {
    if (!id_out) return fail(QRM_E_INVALID, "NULL argument");
    ncclUniqueId id;
    QRM_NCCL(ncclGetUniqueId(&id));
    static_assert(sizeof(ncclUniqueId) == QRM_NCCL_ID_BYTES, "NCCL unique id size");
    memcpy(id_out, &id, sizeof id);
    return QRM_OK;
}

extern "C" int qrm_create_ep(const qrm_layer_desc* desc, int rank, int world, const void* nccl_id, qrm_layer** out) {
    if (!nccl_id) return fail(QRM_E_INVALID, "NULL NCCL id");
    return create_layer(desc, rank, world, nccl_id, out);
}

extern "C" int qrm_ep_transport(qrm_layer* L, int* transport) {
    if (!L || !transport) return fail(QRM_E_INVALID, "NULL argument");
    *transport = L->world == 1 ? QRM_EP_SINGLE : (L->p2p ? QRM_EP_PEER : QRM_EP_NCCL);
    return QRM_OK;
}

extern "C" int qrm_layer_get_desc(qrm_layer* L, qrm_layer_desc* desc) {
    if (!L || !desc) return fail(QRM_E_INVALID, "NULL argument");
    *desc = L->desc;
    return QRM_OK;
}

extern "C" int qrm_expert_range(qrm_layer* L, int* first, int* count) {
    if (!L || !first || !count) return fail(QRM_E_INVALID, "NULL argument");
    *first = L->first_expert;
    *count = L->n_local;
    return QRM_OK;
}

bool ep_p2p_requested() {
    const char* v = getenv("QRM_EP_P2P");
    return !(v && v[0] == '0');
}

// Every rank gathers every rank's 128-byte record through the layer's NCCL
// communicator (in place in L->xch) and copies the records to `all`.
static int ep_allgather128(qrm_layer* L, const void* mine, std::vector<char>& all) {
    const int G = L->world;
    QRM_CUDA(cudaMemcpy(L->xch + 128 * L->rank, mine, 128, cudaMemcpyHostToDevice));
    QRM_NCCL(ncclAllGather(L->xch + 128 * L->rank, L->xch, 128, ncclUint8, L->comm, L->stream));
    QRM_CUDA(cudaStreamSynchronize(L->stream));
    all.resize((size_t)128 * G);
    QRM_CUDA(cudaMemcpy(all.data(), L->xch, (size_t)128 * G, cudaMemcpyDeviceToHost));
    return QRM_OK;
}

// Peer-memory mode: map every other rank's mailbox (CUDA IPC; NVLink peer
// access) when all ranks can, else keep the NCCL exchanges.  All ranks take
// the same decision.
static int ep_open_peers(qrm_layer* L) {
    const int G = L->world;
    char mine[128] = {};
    int ok = ep_p2p_requested() ? 1 : 0;
    cudaIpcMemHandle_t h{};
    static_assert(sizeof(cudaIpcMemHandle_t) <= 120, "IPC handle size");
    if (ok && cudaIpcGetMemHandle(&h, L->mbox) != cudaSuccess) {
        cudaGetLastError();
        ok = 0;
    }
    memcpy(mine, &h, sizeof h);
    memcpy(mine + 120, &ok, sizeof ok);
    std::vector<char> all;
    int rc = ep_allgather128(L, mine, all);
    if (rc) return rc;
    int all_ok = 1;
    for (int q = 0; q < G; q++) {
        int v;
        memcpy(&v, all.data() + 128 * q + 120, sizeof v);
        all_ok &= v;
    }
    std::vector<unsigned long long> base(G, 0);
    base[L->rank] = (unsigned long long)L->mbox;
    int opened = all_ok;
    for (int q = 0; q < G && opened; q++) {
        if (q == L->rank) continue;
        cudaIpcMemHandle_t hq;
        memcpy(&hq, all.data() + 128 * q, sizeof hq);
        void* ptr = nullptr;
        if (cudaIpcOpenMemHandle(&ptr, hq, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            cudaGetLastError();
            opened = 0;
            break;
        }
        L->peer_open.push_back(ptr);
        base[q] = (unsigned long long)ptr;
    }
    // second round: every rank mapped every peer
    memset(mine, 0, sizeof mine);
    memcpy(mine, &opened, sizeof opened);
    rc = ep_allgather128(L, mine, all);
    if (rc) return rc;
    int every = 1;
    for (int q = 0; q < G; q++) {
        int v;
        memcpy(&v, all.data() + 128 * q, sizeof v);
        every &= v;
    }
    if (!every) {
        for (void* p : L->peer_open) cudaIpcCloseMemHandle(p);
        L->peer_open.clear();
        return QRM_OK;
    }
    QRM_CUDA(cudaMemcpy(L->peer_base, base.data(), sizeof(unsigned long long) * G, cudaMemcpyHostToDevice));
    L->p2p = true;
    return QRM_OK;
}

// The tcgen05 grouped path (umma.cu): usable when every expert matrix is in
// the tiled layout in a format pair it has, the gate/up rows come in blocks of
// 64 and the down rows in blocks of 128, and a batch can reach the group size
// it is used from.  Buffers for the largest batch are allocated here.
static int umma_setup(qrm_layer* L) {
    const qrm_layer_desc& D = L->desc;
    const int d = D.d_model, f = D.expert_ffn, E = D.n_experts, k = L->k;
    if (const char* e = getenv("QRM_UMMA")) L->umma_mode = atoi(e) > 0 ? 1 : 0;
    if (const char* e = getenv("QRM_UMMA_MIN_TPE")) L->umma_min_tpe = std::max(1, atoi(e));
    const long long Tx = (long long)D.max_tokens * L->world, Tk = Tx * k;
    const bool sh = L->shared_enabled;
    const int fsh = sh ? D.fmt_sh_gate : -1, fshd = sh ? D.fmt_sh_down : -1;
    const bool fmts = qrm::umma_pair(D.fmt_gate, fsh) && qrm::umma_pair(D.fmt_down, fshd) &&
                      (!sh || (D.fmt_sh_gate == D.fmt_sh_up));
    const bool shapes = umma_shapes(d, f) && layer_tiled(D.fmt_gate, d, f, true) && layer_tiled(D.fmt_down, d, f, false) &&
                        (!sh || (layer_tiled(D.fmt_sh_gate, d, f, true) && layer_tiled(D.fmt_sh_down, d, f, false)));
    L->umma_forced_gu = umma_only_format(D.fmt_gate) || (sh && umma_only_format(D.fmt_sh_gate));
    L->umma_forced_dn = umma_only_format(D.fmt_down) || (sh && umma_only_format(D.fmt_sh_down));
    const bool forced = L->umma_forced_gu || L->umma_forced_dn;
    if (forced && (!fmts || !shapes))
        return fail(QRM_E_FORMAT, "this combination of Q6_K / TRI expert formats and shapes has no kernel");
    const bool reach = forced || L->umma_mode == 1 ||
                       (L->umma_mode != 0 && (Tk >= (long long)L->umma_min_tpe * E || (sh && Tx >= L->umma_min_shared)));
    if (!fmts || !shapes || !reach) return QRM_OK;
    const long long rows = Tk + (sh ? Tx : 0);
    L->umma_cap = qrm::umma_item_cap(L->n_local, Tk, sh ? Tx : 0, f / 64, d / 128);
    if (cudaMalloc(&L->act16, sizeof(__half) * rows * d) != cudaSuccess ||
        cudaMalloc(&L->h16, sizeof(__half) * rows * f) != cudaSuccess ||
        cudaMalloc(&L->umma_items, (size_t)qrm::kUmmaItemBytes * 2 * L->umma_cap) != cudaSuccess ||
        cudaMalloc(&L->umma_count, sizeof(int32_t) * 2) != cudaSuccess)
        return fail(QRM_E_NOMEM, "grouped-path buffers (%lld activation rows)", rows);
    // rows past a batch's end are read as padding: start them at zero
    QRM_CUDA(cudaMemset(L->act16, 0, sizeof(__half) * rows * d));
    QRM_CUDA(cudaMemset(L->h16, 0, sizeof(__half) * rows * f));
    QRM_CUDA(cudaMemset(L->umma_count, 0, sizeof(int32_t) * 2));
    if (qrm::umma_encode_map(&L->act_map, L->act16, rows, d) != 0 || qrm::umma_encode_map(&L->h_map, L->h16, rows, f) != 0)
        return fail(QRM_E_CUDA, "tensor map encoding failed");
    L->umma_ok = true;
    return QRM_OK;
}

static int create_layer(const qrm_layer_desc* desc, int rank, int world, const void* nccl_id, qrm_layer** out,
                        uint8_t* ext_slab) {
    if (!out) return fail(QRM_E_INVALID, "out is NULL");
    *out = nullptr;
    int rc = check_desc(desc);
    if (rc) return rc;
    if (world < 1 || rank < 0 || rank >= world) return fail(QRM_E_INVALID, "rank %d of world %d", rank, world);
    if (desc->n_experts % world) return fail(QRM_E_INVALID, "n_experts %d is not a multiple of world %d", desc->n_experts, world);
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) return fail(QRM_E_CUDA, "no CUDA device");
    if (desc->device < 0 || desc->device >= ndev) return fail(QRM_E_INVALID, "device %d out of range", desc->device);
    cudaDeviceProp prop;
    QRM_CUDA(cudaGetDeviceProperties(&prop, desc->device));
    if (prop.major != 10) return fail(QRM_E_CUDA, "device %d is sm_%d%d; libqrmoe is built for sm_100a", desc->device, prop.major, prop.minor);
    QRM_CUDA(cudaSetDevice(desc->device));
    // the give-up limit of the bounded waits on this device (both units)
    if (const char* e = getenv("QRM_WAIT_LIMIT_US")) {
        const uint64_t ns = (uint64_t)std::max(1LL, atoll(e)) * 1000ull;
        QRM_CUDA(qrm::set_wait_limit_here(ns));
        QRM_CUDA(qrm::umma_set_wait_limit(ns));
    }
    qrm_layer* L = new qrm_layer();
    L->desc = *desc;
    L->k = std::min(desc->n_active, 8);
    L->world = world;
    L->rank = rank;
    L->n_local = desc->n_experts / world;
    L->first_expert = rank * L->n_local;
    L->shared_enabled = desc->moe_sigmoid && desc->n_shared > 0;
    L->sm_count = prop.multiProcessorCount;
    auto bail = [&](int code) { free_layer(L); return code; };
    if (cudaStreamCreateWithFlags(&L->stream, cudaStreamNonBlocking) != cudaSuccess)
        return bail(fail(QRM_E_CUDA, "stream creation failed"));
    const int E = desc->n_experts, d = desc->d_model, f = desc->expert_ffn;
    // slab for all matrices this layer holds
    L->mats.assign((size_t)(E + 1) * 3, qrm::MatDev{});
    L->mat_bytes.assign((size_t)(E + 1) * 3, 0);
    L->uploaded.assign((size_t)(E + 1) * 3, 0);
    size_t total = 0;
    std::vector<size_t> off((size_t)(E + 1) * 3, 0);
    for (int e = 0; e <= E; e++) {
        bool sh = e == E;
        if (sh && !L->shared_enabled) continue;
        if (!sh && (e < L->first_expert || e >= L->first_expert + L->n_local)) continue;
        for (int w = 0; w < 3; w++) {
            int fmt = sh ? (&desc->fmt_sh_gate)[w] : (&desc->fmt_gate)[w];
            int rows = w == 2 ? d : f, cols = w == 2 ? f : d;
            int64_t nb = tensor_bytes(fmt, rows, cols);
            size_t i = (size_t)e * 3 + w;
            off[i] = total;
            L->mat_bytes[i] = (size_t)nb;
            int bs, bb;
            qrm::block_spec(fmt, &bs, &bb);
            L->mats[i] = qrm::MatDev{nullptr, fmt, rows, cols, 0, (int64_t)rows * cols / bs};
            total += ((size_t)nb + 255) / 256 * 256;
        }
    }
    L->slab_bytes = total;
    if (ext_slab) {
        L->slab = ext_slab;
        L->slab_owned = false;
    } else if (cudaMalloc(&L->slab, total) != cudaSuccess) {
        return bail(fail(QRM_E_NOMEM, "cannot allocate %zu bytes of expert weights", total));
    }
    for (size_t i = 0; i < L->mats.size(); i++)
        if (L->mat_bytes[i]) L->mats[i].base = L->slab + off[i];
    if (cudaMalloc(&L->mats_dev, sizeof(qrm::MatDev) * L->mats.size()) != cudaSuccess ||
        cudaMemcpy(L->mats_dev, L->mats.data(), sizeof(qrm::MatDev) * L->mats.size(), cudaMemcpyHostToDevice) != cudaSuccess)
        return bail(fail(QRM_E_NOMEM, "matrix table allocation failed"));
    if (cudaMalloc(&L->norm_w, sizeof(float) * d) != cudaSuccess || cudaMalloc(&L->router, sizeof(float) * (size_t)E * d) != cudaSuccess ||
        cudaMalloc(&L->router_lm, sizeof(float) * (size_t)E * 8 * qrm::route_lane_pitch(d)) != cudaSuccess ||
        cudaMalloc(&L->router_bias, sizeof(float) * E) != cudaSuccess || cudaMalloc(&L->offset, sizeof(float) * E) != cudaSuccess)
        return bail(fail(QRM_E_NOMEM, "router allocation failed"));
    // the expert stages of an expert-parallel layer run over every rank's tokens
    rc = alloc_work(L, desc->max_tokens * world);
    if (rc) return bail(rc);
    L->cap_T = desc->max_tokens;
    if (world > 1) {
        const size_t T = desc->max_tokens, G = world, k = L->k;
        auto up = [](size_t b) { return (b + 255) / 256 * 256; };
        L->mb.rec_flag = 0;
        L->mb.out_flag = (long long)(4 * G);
        L->mb.xn = (long long)up(8 * G);
        L->mb.idx = L->mb.xn + (long long)up(sizeof(float) * G * T * d);
        L->mb.y = L->mb.idx + (long long)up(sizeof(int32_t) * G * T * k);
        const size_t mbox_bytes = (size_t)L->mb.y + sizeof(float) * T * k * d;
        if (cudaMalloc(&L->mbox, mbox_bytes) != cudaSuccess ||
            cudaMalloc(&L->peer_base, sizeof(unsigned long long) * G) != cudaSuccess ||
            cudaMalloc(&L->ep_state, sizeof(uint32_t) * (1 + 2 * G)) != cudaSuccess ||
            cudaMalloc(&L->xch, 128 * G) != cudaSuccess)
            return bail(fail(QRM_E_NOMEM, "expert-parallel buffers"));
        L->xn_all = reinterpret_cast<float*>(L->mbox + L->mb.xn);
        L->idx_all = reinterpret_cast<int32_t*>(L->mbox + L->mb.idx);
        // flags and counters start at zero before any peer can see the mailbox
        if (cudaMemset(L->mbox, 0, mbox_bytes) != cudaSuccess ||
            cudaMemset(L->ep_state, 0, sizeof(uint32_t) * (1 + 2 * G)) != cudaSuccess ||
            cudaMemset(L->xch, 0, 128 * G) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess)
            return bail(fail(QRM_E_CUDA, "expert-parallel buffer initialisation"));
        ncclUniqueId id;
        memcpy(&id, nccl_id, sizeof id);
        ncclResult_t nr = ncclCommInitRank(&L->comm, world, id, rank);
        if (nr != ncclSuccess) return bail(fail(QRM_E_NCCL, "ncclCommInitRank: %s", ncclGetErrorString(nr)));
        rc = ep_open_peers(L);
        if (rc) return bail(rc);
        if (L->p2p) {
            L->yrecv = reinterpret_cast<float*>(L->mbox + L->mb.y);
        } else {
            // NCCL: gathered records, one send and one receive block per peer
            if (cudaMalloc(&L->rec_own, sizeof(float) * T * (d + 2 * k)) != cudaSuccess ||
                cudaMalloc(&L->rec_all, sizeof(float) * G * T * (d + 2 * k)) != cudaSuccess ||
                cudaMalloc(&L->ysend, sizeof(float) * G * T * k * d) != cudaSuccess ||
                cudaMalloc(&L->yrecv_nccl, sizeof(float) * G * T * k * d) != cudaSuccess)
                return bail(fail(QRM_E_NOMEM, "expert-parallel NCCL buffers"));
            L->yrecv = L->yrecv_nccl;
        }
    }
    rc = umma_setup(L);
    if (rc) return bail(rc);
    // kernels with large dynamic shared memory
    if (cudaFuncSetAttribute(qrm::route_small_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) != cudaSuccess ||
        cudaFuncSetAttribute(qrm::route_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024) != cudaSuccess ||
        cudaFuncSetAttribute(qrm::dispatch_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) != cudaSuccess ||
        cudaFuncSetAttribute(qrm::topk_dispatch_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)qrm::topk_dispatch_smem(256, qrm::kFusedTopkMaxT)) != cudaSuccess ||
        cudaFuncSetAttribute(qrm::topk_dispatch_kernel<qrm::kMaxE / 32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)qrm::topk_dispatch_smem(qrm::kMaxE, qrm::kFusedTopkMaxT)) != cudaSuccess ||
        cudaFuncSetAttribute(qrm::rmsnorm_row_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024) != cudaSuccess ||
        !lm_tiles_setup())
        return bail(fail(QRM_E_CUDA, "kernel attribute"));
    *out = L;
    return QRM_OK;
}

extern "C" void qrm_destroy(qrm_layer* layer) { free_layer(layer); }

extern "C" int qrm_upload_norm(qrm_layer* L, const float* w) {
    if (!L || !w) return fail(QRM_E_INVALID, "NULL argument");
    clear_graphs(L);
    QRM_CUDA(cudaSetDevice(L->desc.device));
    QRM_CUDA(cudaMemcpy(L->norm_w, w, sizeof(float) * L->desc.d_model, cudaMemcpyHostToDevice));
    L->has_norm = true;
    return QRM_OK;
}

extern "C" int qrm_upload_router(qrm_layer* L, const float* w, const float* bias) {
    if (!L || !w) return fail(QRM_E_INVALID, "NULL argument");
    clear_graphs(L);
    QRM_CUDA(cudaSetDevice(L->desc.device));
    QRM_CUDA(cudaMemcpy(L->router, w, sizeof(float) * (size_t)L->desc.n_experts * L->desc.d_model, cudaMemcpyHostToDevice));
    qrm::router_lane_major_kernel<<<L->sm_count * 4, 256>>>(L->router, L->router_lm, L->desc.n_experts, L->desc.d_model);
    QRM_CUDA(cudaDeviceSynchronize());
    if (bias) QRM_CUDA(cudaMemcpy(L->router_bias, bias, sizeof(float) * L->desc.n_experts, cudaMemcpyHostToDevice));
    L->has_bias = bias != nullptr;
    L->has_router = true;
    return QRM_OK;
}

extern "C" int qrm_upload_logit_offset(qrm_layer* L, const float* offset) {
    if (!L) return fail(QRM_E_INVALID, "NULL layer");
    clear_graphs(L);
    QRM_CUDA(cudaSetDevice(L->desc.device));
    if (offset) QRM_CUDA(cudaMemcpy(L->offset, offset, sizeof(float) * L->desc.n_experts, cudaMemcpyHostToDevice));
    L->has_offset = offset != nullptr;
    return QRM_OK;
}

static int mat_index(qrm_layer* L, int expert, int which, size_t* idx) {
    if (which < 0 || which > 2) return fail(QRM_E_INVALID, "which must be 0 (gate), 1 (up) or 2 (down)");
    const int E = L->desc.n_experts;
    int e;
    if (expert == QRM_SHARED_EXPERT) {
        if (!L->shared_enabled) return fail(QRM_E_INVALID, "this layer has no shared expert (needs moe_sigmoid and n_shared > 0)");
        e = E;
    } else {
        if (expert < 0 || expert >= E) return fail(QRM_E_INVALID, "expert %d out of range [0, %d)", expert, E);
        if (expert < L->first_expert || expert >= L->first_expert + L->n_local)
            return fail(QRM_E_INVALID, "expert %d is not held by this layer", expert);
        e = expert;
    }
    *idx = (size_t)e * 3 + which;
    return QRM_OK;
}

static int upload_common(qrm_layer* L, int expert, int which, int fmt, const void* bytes, size_t nbytes, bool dev) {
    if (!L || !bytes) return fail(QRM_E_INVALID, "NULL argument");
    clear_graphs(L);
    size_t i;
    int rc = mat_index(L, expert, which, &i);
    if (rc) return rc;
    const qrm::MatDev& m = L->mats[i];
    if (fmt != m.fmt)
        return fail(QRM_E_FORMAT, "l.e%d.%s: format %d, layer expects %d", expert, which_name(which), fmt, m.fmt);
    if (nbytes != L->mat_bytes[i])
        return fail(QRM_E_SIZE, "l.e%d.%s: %zu bytes, TensorBytes(%d x %d) = %zu", expert, which_name(which), nbytes,
                    m.rows, m.cols, L->mat_bytes[i]);
    QRM_CUDA(cudaSetDevice(L->desc.device));
    // device bytes may still be in flight on another stream of the caller
    // (the layer's own stream does not order with them): finish all work first
    if (dev) QRM_CUDA(cudaDeviceSynchronize());
    uint8_t* dst = const_cast<uint8_t*>(m.base);
    const bool tiled = layer_tiled(fmt, L->desc.d_model, L->desc.expert_ffn, which != 2);
    if ((fmt == qrm::Q4_K && !tiled) || qrm::is_raw_fmt(fmt)) {
        QRM_CUDA(cudaMemcpyAsync(dst, bytes, nbytes, dev ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, L->stream));
    } else {
        const uint8_t* src = (const uint8_t*)bytes;
        if (!dev) {
            if (L->staging_bytes < nbytes) {
                if (L->staging) cudaFree(L->staging);
                L->staging = nullptr;
                L->staging_bytes = 0;
                if (cudaMalloc(&L->staging, nbytes) != cudaSuccess) return fail(QRM_E_NOMEM, "staging allocation failed");
                L->staging_bytes = nbytes;
            }
            QRM_CUDA(cudaMemcpyAsync(L->staging, bytes, nbytes, cudaMemcpyHostToDevice, L->stream));
            src = L->staging;
        }
        int bs, bb;
        qrm::block_spec(fmt, &bs, &bb);
        long long nb = (long long)(nbytes / bb);
        if (tiled)
            qrm::tile_relayout_kernel<<<L->sm_count * 8, 256, 0, L->stream>>>(fmt, bb, m.cols / 256, src, dst, nb, 1);
        else
            qrm::relayout_kernel<<<L->sm_count * 8, 256, 0, L->stream>>>(fmt, bb, src, dst, nb, 1);
        QRM_CUDA(cudaGetLastError());
    }
    QRM_CUDA(cudaStreamSynchronize(L->stream));
    // a streamed layer of a stack keeps its weights in a host image of its slab
    if (L->image) QRM_CUDA(cudaMemcpy(L->image + (m.base - L->slab), m.base, L->mat_bytes[i], cudaMemcpyDeviceToHost));
    L->uploaded[i] = 1;
    return QRM_OK;
}

extern "C" int qrm_upload_expert(qrm_layer* L, int expert, int which, int fmt, const void* bytes, size_t nbytes) {
    return upload_common(L, expert, which, fmt, bytes, nbytes, false);
}
extern "C" int qrm_upload_expert_device(qrm_layer* L, int expert, int which, int fmt, const void* bytes_dev, size_t nbytes) {
    return upload_common(L, expert, which, fmt, bytes_dev, nbytes, true);
}

extern "C" int qrm_download_expert(qrm_layer* L, int expert, int which, void* bytes, size_t nbytes) {
    if (!L || !bytes) return fail(QRM_E_INVALID, "NULL argument");
    size_t i;
    int rc = mat_index(L, expert, which, &i);
    if (rc) return rc;
    if (!L->uploaded[i]) return fail(QRM_E_STATE, "l.e%d.%s was never uploaded", expert, which_name(which));
    if (nbytes != L->mat_bytes[i]) return fail(QRM_E_SIZE, "buffer is %zu bytes, tensor is %zu", nbytes, L->mat_bytes[i]);
    const qrm::MatDev& m = L->mats[i];
    QRM_CUDA(cudaSetDevice(L->desc.device));
    const bool tiled = layer_tiled(m.fmt, L->desc.d_model, L->desc.expert_ffn, which != 2);
    // a streamed layer's bytes are in its host image (its slot holds whichever
    // layer ran last)
    const uint8_t* img = L->image ? L->image + (m.base - L->slab) : nullptr;
    if ((m.fmt == qrm::Q4_K && !tiled) || qrm::is_raw_fmt(m.fmt)) {
        if (img) memcpy(bytes, img, nbytes);
        else QRM_CUDA(cudaMemcpy(bytes, m.base, nbytes, cudaMemcpyDeviceToHost));
        return QRM_OK;
    }
    uint8_t* tmp = nullptr;
    QRM_CUDA(cudaMalloc(&tmp, 2 * nbytes));
    const uint8_t* src = m.base;
    if (img) {
        cudaMemcpy(tmp + nbytes, img, nbytes, cudaMemcpyHostToDevice);
        src = tmp + nbytes;
    }
    int bs, bb;
    qrm::block_spec(m.fmt, &bs, &bb);
    if (tiled)
        qrm::tile_relayout_kernel<<<L->sm_count * 8, 256, 0, L->stream>>>(m.fmt, bb, m.cols / 256, src, tmp,
                                                                         (long long)(nbytes / bb), 0);
    else
        qrm::relayout_kernel<<<L->sm_count * 8, 256, 0, L->stream>>>(m.fmt, bb, src, tmp, (long long)(nbytes / bb), 0);
    cudaError_t e1 = cudaStreamSynchronize(L->stream);
    cudaError_t e2 = cudaMemcpy(bytes, tmp, nbytes, cudaMemcpyDeviceToHost);
    cudaFree(tmp);
    if (e1 != cudaSuccess || e2 != cudaSuccess) return fail(QRM_E_CUDA, "download failed: %s", cudaGetErrorString(e1 != cudaSuccess ? e1 : e2));
    return QRM_OK;
}

static int forward_checks(qrm_layer* L, int T, int flags) {
    if (T <= 0) return fail(QRM_E_INVALID, "T must be positive");
    if (T > L->cap_T) return fail(QRM_E_CAPACITY, "T = %d exceeds max_tokens = %d", T, L->cap_T);
    if (!L->has_router) return fail(QRM_E_STATE, "tensor l.router was never uploaded");
    if ((flags & QRM_APPLY_NORM) && !L->has_norm) return fail(QRM_E_STATE, "tensor l.ffn_norm was never uploaded");
    if (flags & ~(QRM_APPLY_NORM | QRM_ADD_RESIDUAL)) return fail(QRM_E_INVALID, "unknown flags 0x%x", flags);
    const int E = L->desc.n_experts;
    for (int e = L->first_expert; e < L->first_expert + L->n_local; e++)
        for (int w = 0; w < 3; w++)
            if (!L->uploaded[(size_t)e * 3 + w]) return fail(QRM_E_STATE, "tensor l.e%d.%s was never uploaded", e, which_name(w));
    if (L->shared_enabled) {
        int n = L->uploaded[(size_t)E * 3] + L->uploaded[(size_t)E * 3 + 1] + L->uploaded[(size_t)E * 3 + 2];
        if (n != 0 && n != 3) return fail(QRM_E_STATE, "shared expert is only partly uploaded");
    }
    return QRM_OK;
}

static qrm::EpPeers ep_peers(const qrm_layer* L) {
    qrm::EpPeers p{};
    p.base = L->peer_base;
    p.mb = L->mb;
    p.epoch = L->ep_state;
    p.cnt = L->ep_state + 1;
    p.err = &L->sched->err;
    p.G = L->world;
    p.rank = L->rank;
    return p;
}

static int launch_forward(qrm_layer* L, const float* x, int T, int flags, float* out, int32_t* topk_idx,
                          float* topk_w, cudaStream_t s) {
    const qrm_layer_desc& D = L->desc;
    const int d = D.d_model, E = D.n_experts, f = D.expert_ffn, k = L->k;
    const bool shared = L->shared_enabled && L->uploaded[(size_t)E * 3];
    const bool prof = L->profiling;
    int nl = 0;   // kernel launches of this forward
    // expert parallelism: the expert stages run over every rank's tokens
    const bool ep = L->world > 1;
    // stage boundaries: event i_single of a single-GPU forward, i_ep of an
    // expert-parallel one (-1: not a boundary there)
    auto mark = [&](int i_single, int i_ep) {
        const int i = ep ? i_ep : i_single;
        if (prof && i >= 0) cudaEventRecordWithFlags(L->ev[i], s, cudaEventRecordExternal);
    };
    mark(0, 0);
    // 1. RMSNorm + router logits, 2. top-k, 3. dispatch
    const float* xn = L->xn;
    qrm::TopkParams tp{L->logits, L->has_bias ? L->router_bias : nullptr, topk_idx, topk_w, T, E, k,
                       D.moe_sigmoid ? 1 : 0, D.routed_scale};
    qrm::DispatchParams dp{topk_idx, L->perm, L->inv_perm, L->pos_tok, L->slot_info, L->offsets, L->active, L->sched, T, k, E,
                           L->first_expert, L->n_local, shared ? 1 : 0};
    dp.T_sh = T;
    qrm::RouteParams rp{x, L->norm_w, L->router, L->has_offset ? L->offset : nullptr, L->xn, L->logits, T, d, E,
                        (flags & QRM_APPLY_NORM) ? 1 : 0, D.rms_eps};
    if (T <= qrm::route_fused_max_tokens(d, E) && (reinterpret_cast<uintptr_t>(x) & 15) == 0) {
        // one launch: every CTA its experts' logits, the last CTA top-k + dispatch
        const int grid = (E + qrm::kRouteEPC - 1) / qrm::kRouteEPC;
        qrm::RouteFusedParams fp{rp, L->router_lm, tp, dp};
        nl++;
        qrm::route_fused_kernel<<<grid, qrm::kRouteThreads, qrm::route_fused_smem(d, T, E), s>>>(fp);
        QRM_CUDA(cudaGetLastError());
        mark(1, -1);
        mark(2, -1);
        mark(3, 1);
    } else {
        if (T <= qrm::route_small_max_tokens(d)) {
            int grid = (E + qrm::kRouteEPC - 1) / qrm::kRouteEPC;
            nl++;
            qrm::route_small_kernel<<<grid, qrm::kRouteThreads, qrm::route_small_smem(d, T), s>>>(rp);
        } else {
            if (flags & QRM_APPLY_NORM) {
                nl++;
                if ((reinterpret_cast<uintptr_t>(x) & 15) == 0 && d % 4 == 0 &&
                    qrm::rmsnorm_row_smem(d) <= 200 * 1024)
                    qrm::rmsnorm_row_kernel<<<T, qrm::kNormRowThreads, qrm::rmsnorm_row_smem(d), s>>>(
                        x, L->norm_w, L->xn, d, D.rms_eps);
                else
                    qrm::rmsnorm_kernel<<<(T + 7) / 8, 256, 0, s>>>(x, L->norm_w, L->xn, T, d, D.rms_eps);
            } else {
                xn = x;
            }
            nl++;
            launch_logits_lm(xn, L->router_lm, L->has_offset ? L->offset : nullptr, L->logits, T, d, E, L->sm_count, s);
        }
        QRM_CUDA(cudaGetLastError());
        mark(1, -1);
        // top-k and dispatch (one single-CTA kernel for T <= 32)
        if (T <= qrm::kFusedTopkMaxT) {
            mark(2, -1);
            nl++;
            const size_t sm = qrm::topk_dispatch_smem(E, T);
            if (E <= 256) qrm::topk_dispatch_kernel<8><<<1, qrm::kDispatchThreads, sm, s>>>(dp, tp);
            else qrm::topk_dispatch_kernel<qrm::kMaxE / 32><<<1, qrm::kDispatchThreads, sm, s>>>(dp, tp);
        } else {
            nl += 2;
            if (E <= 256) qrm::topk_kernel<8><<<(T + 3) / 4, 128, 0, s>>>(tp);
            else qrm::topk_kernel<qrm::kMaxE / 32><<<(T + 3) / 4, 128, 0, s>>>(tp);
            QRM_CUDA(cudaGetLastError());
            mark(2, -1);
            qrm::dispatch_kernel<<<1, qrm::kDispatchThreads, qrm::dispatch_smem(E), s>>>(dp);
        }
        QRM_CUDA(cudaGetLastError());
        mark(3, 1);
    }
    L->last_xn = xn;
    const int G = L->world;
    int Tx = T;
    const float* xs = xn;
    if (ep) {
        Tx = G * T;
        xs = L->xn_all;
    }
    // the shared expert runs for this rank's own tokens only: rows
    // [sh_row0, sh_row0 + T) of xs (each rank's rows sit at rank*T)
    const int Tsh = T;
    const int sh_row0 = ep ? L->rank * T : 0;
    if (ep && L->p2p) {
        // records straight into every rank's mailbox; the dispatch waits for all of them
        const qrm::EpPeers pe = ep_peers(L);
        // blocks per destination: one per 1024 float4 of the rows, up to two
        // waves of the GPU over all destinations (large batches move tens of MB)
        const int nb = (int)std::max<long long>(
            1, std::min<long long>(((long long)T * d / 4 + 1023) / 1024, std::max(16, 2 * L->sm_count / G)));
        qrm::ep_push_records_kernel<<<G * nb, 256, 0, s>>>(xn, topk_idx, T, d, k, E / G, pe);
        QRM_CUDA(cudaGetLastError());
        qrm::DispatchParams dpx{L->idx_all, L->perm, L->inv_perm, L->pos_tok, L->slot_info, L->offsets, L->active, L->sched,
                                Tx, k, E, L->first_expert, L->n_local, shared ? 1 : 0,
                                reinterpret_cast<const uint32_t*>(L->mbox + L->mb.rec_flag), L->ep_state, G, Tsh, 1};
        qrm::dispatch_kernel<<<1, qrm::kDispatchThreads, qrm::dispatch_smem(E), s>>>(dpx);
        QRM_CUDA(cudaGetLastError());
        nl += 2;
        mark(-1, 2);
    } else if (ep) {
        // (normalised token, top-k) records of every rank
        const int W = d + 2 * k;
        const long long nrec = (long long)T * W;
        int grid = (int)std::min<long long>((nrec + 255) / 256, (long long)L->sm_count * 8);
        qrm::ep_pack_records_kernel<<<grid, 256, 0, s>>>(xn, topk_idx, topk_w, T, d, k, L->rec_own);
        QRM_CUDA(cudaGetLastError());
        QRM_NCCL(ncclAllGather(L->rec_own, L->rec_all, (size_t)nrec, ncclFloat32, L->comm, s));
        grid = (int)std::min<long long>(((long long)Tx * (d + k) + 255) / 256, (long long)L->sm_count * 8);
        qrm::ep_unpack_records_kernel<<<grid, 256, 0, s>>>(L->rec_all, Tx, d, k, L->xn_all, L->idx_all);
        QRM_CUDA(cudaGetLastError());
        // dispatch of all ranks' assignments; the active list holds this rank's experts
        qrm::DispatchParams dpx{L->idx_all, L->perm, L->inv_perm, L->pos_tok, L->slot_info, L->offsets, L->active, L->sched,
                                Tx, k, E, L->first_expert, L->n_local, shared ? 1 : 0};
        dpx.T_sh = Tsh;
        dpx.local_only = 1;
        qrm::dispatch_kernel<<<1, qrm::kDispatchThreads, qrm::dispatch_smem(E), s>>>(dpx);
        QRM_CUDA(cudaGetLastError());
        nl += 3;
        mark(-1, 2);
    }
    // 4. gate/up (+ SwiGLU) and 5. down
    // each stage takes the tcgen05 grouped path for large groups, and always
    // for the formats that have no other kernel in the tiled layout
    const bool large = L->umma_ok && (L->umma_mode == 1 ||
                                      (L->umma_mode != 0 && ((long long)Tx * k >= (long long)L->umma_min_tpe * E ||
                                                             (shared && Tx >= L->umma_min_shared))));
    const bool u_gu = L->umma_ok && (large || L->umma_forced_gu);
    const bool u_dn = L->umma_ok && (large || L->umma_forced_dn);
    const int Tk = Tx * k;
    bool ep_stored = false;   // the down kernel stored the output rows into the owners' mailboxes
    if (u_gu || u_dn) {
        // work lists of both stages from the dispatch's slot table; f16
        // activations in dispatch order for a grouped gate/up
        if (u_gu)
            QRM_CUDA(qrm::umma_gather(xs, xs + (size_t)sh_row0 * d, L->pos_tok, Tk, shared ? Tsh : 0, d, L->act16,
                                      L->sm_count, s));
        QRM_CUDA(qrm::umma_plan(L->slot_info, &L->sched->n_active, shared ? 1 : 0, Tk, f / 64, d / 128, E,
                                L->umma_items, L->umma_count, L->umma_items + L->umma_cap, L->umma_count + 1,
                                (int)L->umma_cap, s));
        nl += u_gu ? 2 : 1;
    }
    const int nt = pick_nt(Tx);
    const float limit = D.moe_sigmoid ? D.swiglu_limit : 0.f;  // MoeFfn / LegacyMoeInto use plain SiLU
    const bool same_fmt = !shared || (D.fmt_sh_gate == D.fmt_gate && D.fmt_sh_down == D.fmt_down);
    bool combined = false;
    for (int stage = 0; stage < 2; stage++) {
        const bool gu = stage == 0;
        const float ulimit = D.moe_sigmoid ? D.swiglu_limit : 0.f;
        if (gu && u_gu) {
            cudaError_t e = qrm::umma_expert(D.fmt_gate, shared ? D.fmt_sh_gate : -1, true, L->act_map, L->mats_dev,
                                             L->umma_items, L->umma_count, d, f, Tk, ulimit, L->h16, nullptr, nullptr,
                                             &L->sched->err, L->sm_count, s);
            if (e != cudaSuccess) return fail(QRM_E_CUDA, "grouped gate/up launch: %s", cudaGetErrorString(e));
            nl++;
            mark(4, 3);
            continue;
        }
        if (!gu && u_dn != u_gu) {
            // the stages took different paths: hand the SwiGLU outputs over
            // (f32 h / hs of the decode kernels <-> f16 rows of the grouped one)
            QRM_CUDA(qrm::umma_convert_h(L->h, shared ? L->hs : nullptr, Tk, shared ? Tsh : 0, f, L->h16, u_dn ? 1 : 0,
                                         L->sm_count, s));
            nl++;
        }
        if (!gu && u_dn) {
            cudaError_t e = qrm::umma_expert(D.fmt_down, shared ? D.fmt_sh_down : -1, false, L->h_map, L->mats_dev,
                                             L->umma_items + L->umma_cap, L->umma_count + 1, f, d, Tk, 0.f, nullptr,
                                             L->y, L->ys, &L->sched->err, L->sm_count, s);
            if (e != cudaSuccess) return fail(QRM_E_CUDA, "grouped down launch: %s", cudaGetErrorString(e));
            nl++;
            mark(5, 4);
            continue;
        }
        // activation tables for the integer tensor-core kernel
        const int frs = gu ? D.fmt_gate : D.fmt_down, fss = gu ? D.fmt_sh_gate : D.fmt_sh_down;
        const int rows_s = gu ? f : d, cols_s = gu ? d : f;
        const bool want_tab = imma_usable(frs, rows_s, cols_s, gu) || (shared && imma_usable(fss, rows_s, cols_s, gu));
        qrm::GemvParams gp{};
        gp.xtab = want_tab ? (gu ? L->xtab_gu : L->xtab_dn) : nullptr;
        gp.xtab_stride = qrm::xtab_stride(cols_s);
        gp.xtab_shared_base = gu ? sh_row0 : Tx * k;
        gp.xtab_rows = gu ? Tx : Tx * k + (shared ? Tsh : 0);
        gp.mats = L->mats_dev;
        gp.active = L->active;
        gp.offsets = L->offsets;
        gp.perm = L->perm;
        gp.pos_tok = L->pos_tok;
        gp.slot_info = L->slot_info;
        gp.n_active = &L->sched->n_active;
        gp.x_routed = gu ? xs : L->h;
        gp.x_shared = gu ? xs + (size_t)sh_row0 * d : L->hs;
        gp.out_routed = gu ? L->h : L->y;
        gp.out_shared = gu ? L->hs : L->ys;
        gp.T = Tx;
        gp.T_sh = Tsh;
        gp.k = k;
        gp.E = E;
        gp.rows = gu ? f : d;
        gp.cols = gu ? d : f;
        gp.tiles = (gp.rows + (gu ? kRGateUp : kRDown) - 1) / (gu ? kRGateUp : kRDown);
        gp.limit = limit;
        gp.routed_by_token = gu ? 1 : 0;
        gp.has_shared = shared ? 1 : 0;
        const int fr = gu ? D.fmt_gate : D.fmt_down;
        const int fs = gu ? D.fmt_sh_gate : D.fmt_sh_down;
        gp.pdl = (!prof && (L->pdl & (gu ? 1 : 2))) ? (gu ? 1 : 2) : 0;   // profiling events sit between the launches

        // routed + shared expert in one integer-kernel launch when the pair of
        // formats has one
        StreamSel sp;
        gp.mode = 0;
        const bool pair = want_tab && shared && !same_fmt && imma_pair_supported(fr, fs) && stream_select(fr, fs, gu, Tx, gp, L->sm_count, &sp);
        if (want_tab) {
            // the kernels quantise resident tables themselves when every
            // integer-kernel launch of this stage keeps them resident
            bool in_kernel;
            if (pair) {
                in_kernel = sp.cfg.res_rows > 0;
            } else {
                StreamSel sr, ss;
                const bool ur = imma_usable(fr, gp.rows, gp.cols, gu);
                const bool us = shared && !same_fmt && imma_usable(fs, gp.rows, gp.cols, gu);
                gp.mode = same_fmt ? 0 : 1;
                const bool pr = ur && stream_select(fr, same_fmt && shared ? fr : -1, gu, Tx, gp, L->sm_count, &sr);
                gp.mode = 2;
                const bool ps = us && stream_select(-1, fs, gu, Tx, gp, L->sm_count, &ss);
                gp.mode = 0;
                in_kernel = (ur || us) && (!ur || (pr && sr.cfg.res_rows > 0)) && (!us || (ps && ss.cfg.res_rows > 0));
            }
            if (in_kernel) {
                gp.xq_a = gu ? xs : L->h;
                gp.xq_b = gu ? xs : L->hs;
                gp.xq_split = gu ? Tx : Tx * k;
            } else {
                int rc;
                if (gu) {
                    rc = launch_xquant(xs, d, Tx, L->xtab_gu, s);
                    nl++;
                } else {
                    // routed rows, then the shared rows right after them
                    rc = launch_xquant(L->h, f, Tx * k + (shared ? Tsh : 0), L->xtab_dn, s, L->hs, Tx * k);
                    nl++;
                }
                if (rc) return rc;
            }
        }
        // expert parallelism over peer memory: the streaming down kernel stores
        // the routed output rows into their owners' mailboxes and raises the
        // output flags itself
        if (!gu && ep && L->p2p && imma_usable(fr, gp.rows, gp.cols, false)) {
            gp.ep_base = L->peer_base;
            gp.ep_y = L->mb.y;
            gp.ep_flag = L->mb.out_flag;
            gp.ep_epoch = L->ep_state;
            gp.ep_cnt = L->ep_state + 1 + G;
            gp.ep_G = G;
            gp.ep_rank = L->rank;
            gp.ep_T = T;
            ep_stored = true;
        }
        if (pair) {
            gp.mode = 0;
            gp.ctr = &L->sched->ctr[gu ? 0 : 2];
            int rc = launch_stream_pair(gu, Tx, gp, L->sm_count, &L->sched->err, s);
            if (rc) return rc;
            nl++;
        } else if (same_fmt) {
            gp.mode = 0;
            gp.ctr = &L->sched->ctr[gu ? 0 : 2];
            int rc = launch_gemv(fr, gu, nt, gp, L->sm_count, &L->sched->err, s);
            if (rc) return rc;
            nl++;
        } else {
            gp.mode = 1;
            gp.ctr = &L->sched->ctr[gu ? 0 : 2];
            int rc = launch_gemv(fr, gu, nt, gp, L->sm_count, &L->sched->err, s);
            if (rc) return rc;
            gp.mode = 2;
            gp.ctr = &L->sched->ctr[gu ? 1 : 3];
            gp.ep_base = nullptr;   // shared rows stay here
            rc = launch_gemv(fs, gu, nt, gp, L->sm_count, &L->sched->err, s);
            if (rc) return rc;
            nl += 2;
        }
        mark(gu ? 4 : 5, gu ? 3 : 4);
    }
    if (ep && L->p2p) {
        // expert output rows straight into the owners' mailboxes; the owner
        // combines in slot order once every holder's rows are in
        const qrm::EpPeers pe = ep_peers(L);
        if (!ep_stored) {
            // grid for the largest possible number of local assignments
            const long long n4 = (long long)Tx * k * (d / 4);
            const int pgrid =
                (int)std::max<long long>(1, std::min<long long>((n4 + 255) / 256, (long long)L->sm_count * 4));
            qrm::ep_push_outputs_kernel<<<pgrid, 256, 0, s>>>(L->y, L->perm, L->offsets + E, T, k, d, pe);
            QRM_CUDA(cudaGetLastError());
            nl++;
        }
        mark(-1, 5);
        const long long m4 = (long long)T * (d / 4);
        const int grid = (int)std::min<long long>((m4 + 255) / 256, (long long)L->sm_count * 16);
        qrm::ep_combine_kernel<<<grid, 256, 0, s>>>((flags & QRM_ADD_RESIDUAL) ? x : nullptr, topk_w, topk_idx, L->yrecv,
                                                    shared ? L->ys : nullptr, T, k, d, E / G, 0, out,
                                                    reinterpret_cast<const uint32_t*>(L->mbox + L->mb.out_flag),
                                                    L->ep_state, G, &L->sched->err);
        QRM_CUDA(cudaGetLastError());
        nl++;
        combined = true;
    } else if (ep) {
        // expert output rows back to the token owners; the owner combines in slot order
        const long long n4 = (long long)Tx * k * (d / 4);
        int grid = (int)std::min<long long>((n4 + 255) / 256, (long long)L->sm_count * 16);
        qrm::ep_pack_outputs_kernel<<<grid, 256, 0, s>>>(L->y, L->inv_perm, L->idx_all, G, T, k, d, L->first_expert,
                                                         L->n_local, L->ysend);
        QRM_CUDA(cudaGetLastError());
        const size_t blk = (size_t)T * k * d;
        QRM_NCCL(ncclGroupStart());
        for (int q = 0; q < G; q++) {
            QRM_NCCL(ncclSend(L->ysend + q * blk, blk, ncclFloat32, q, L->comm, s));
            QRM_NCCL(ncclRecv(L->yrecv + q * blk, blk, ncclFloat32, q, L->comm, s));
        }
        QRM_NCCL(ncclGroupEnd());
        mark(-1, 5);
        const long long m4 = (long long)T * (d / 4);
        grid = (int)std::min<long long>((m4 + 255) / 256, (long long)L->sm_count * 16);
        qrm::ep_combine_kernel<<<grid, 256, 0, s>>>((flags & QRM_ADD_RESIDUAL) ? x : nullptr, topk_w, topk_idx, L->yrecv,
                                                    shared ? L->ys : nullptr, T, k, d, E / G, 1, out, nullptr, nullptr,
                                                    0, nullptr);
        QRM_CUDA(cudaGetLastError());
        nl += 2;
        combined = true;
    }
    // 6. combine (unless the down kernel did it)
    if (!combined) {
        qrm::CombineParams cp{(flags & QRM_ADD_RESIDUAL) ? x : nullptr, L->y, shared ? L->ys : nullptr, L->inv_perm,
                              topk_w, out, T, k, d, topk_idx, &L->sched->err, L->stage_idx, L->stage_w, L->stage_err};
        long long n4 = (long long)T * (d / 4);
        int cgrid = (int)std::min<long long>((n4 + 255) / 256, (long long)L->sm_count * 16);
        QRM_CUDA(launch_k(!prof && (L->pdl & 4), qrm::combine_kernel, dim3(cgrid), dim3(256), 0, s, cp));
        nl++;
    }
    mark(6, 6);
    L->last_T = T;
    L->last_launches = nl;
    L->profiled_last = prof;
    L->last_shared = shared;
    return QRM_OK;
}

// Runs the forward as a CUDA graph (captured once per buffer set, T, flags
// and profiling state; uploads invalidate the cache) launched on `s`.
static int run_forward(qrm_layer* L, const float* x, int T, int flags, float* out, int32_t* idx, float* w,
                       cudaStream_t s) {
    if (L->world > 1 && !ep_graphs_enabled()) {
        // expert-parallel forwards launched directly (QRM_EP_GRAPH=0)
        int rc = launch_forward(L, x, T, flags, out, idx, w, s);
        if (rc) return rc;
        L->last_T = T;
        L->profiled_last = false;
        L->last_xn = L->xn;
        return QRM_OK;
    }
    // expert-parallel graphs hold NCCL calls: they always run on the layer's own
    // buffers (user buffers are copied in and out) so one graph serves every call
    float* user_out = out;
    int32_t* user_idx = idx;
    float* user_w = w;
    const bool ep_bufs = L->world > 1;
    if (ep_bufs) {
        const size_t xb = sizeof(float) * (size_t)T * L->desc.d_model;
        if (x != L->x) QRM_CUDA(cudaMemcpyAsync(L->x, x, xb, cudaMemcpyDeviceToDevice, s));
        x = L->x;
        out = L->out;
        idx = L->topk_idx;
        w = L->topk_w;
    }
    qrm_layer::GraphKey key{T, flags, L->profiling ? 1 : 0};
    const void* ptrs[4] = {x, out, idx, w};
    auto it = L->graphs.find(key);
    const bool same = it != L->graphs.end() && std::equal(ptrs, ptrs + 4, it->second.ptrs);
    if (!same) {
        QRM_CUDA(cudaStreamBeginCapture(L->stream, cudaStreamCaptureModeThreadLocal));
        int rc = launch_forward(L, x, T, flags, out, idx, w, L->stream);
        cudaGraph_t g = nullptr;
        cudaError_t ce = cudaStreamEndCapture(L->stream, &g);
        if (rc) {
            if (g) cudaGraphDestroy(g);
            return rc;
        }
        if (ce != cudaSuccess) return fail(QRM_E_CUDA, "graph capture: %s", cudaGetErrorString(ce));
        bool updated = false;
        if (it != L->graphs.end()) {
            cudaGraphExecUpdateResultInfo info;
            updated = cudaGraphExecUpdate(it->second.exec, g, &info) == cudaSuccess;
            if (!updated) {
                cudaGetLastError();   // clear the update failure; instantiate instead
                cudaGraphExecDestroy(it->second.exec);
                L->graphs.erase(it);
                it = L->graphs.end();
            }
        }
        if (!updated) {
            if (L->graphs.size() >= 32) clear_graphs(L);
            cudaGraphExec_t ex = nullptr;
            ce = cudaGraphInstantiate(&ex, g, 0);
            if (ce != cudaSuccess) {
                cudaGraphDestroy(g);
                return fail(QRM_E_CUDA, "graph instantiate: %s", cudaGetErrorString(ce));
            }
            it = L->graphs.emplace(key, qrm_layer::Graph{}).first;
            it->second.exec = ex;
        }
        cudaGraphDestroy(g);
        it->second.launches = L->last_launches;
        std::copy(ptrs, ptrs + 4, it->second.ptrs);
    }
    QRM_CUDA(cudaGraphLaunch(it->second.exec, s));
    if (ep_bufs) {
        const size_t xb = sizeof(float) * (size_t)T * L->desc.d_model, kb = (size_t)T * L->k;
        if (user_out != out) QRM_CUDA(cudaMemcpyAsync(user_out, out, xb, cudaMemcpyDeviceToDevice, s));
        if (user_idx != idx) QRM_CUDA(cudaMemcpyAsync(user_idx, idx, sizeof(int32_t) * kb, cudaMemcpyDeviceToDevice, s));
        if (user_w != w) QRM_CUDA(cudaMemcpyAsync(user_w, w, sizeof(float) * kb, cudaMemcpyDeviceToDevice, s));
    }
    L->last_T = T;
    L->last_launches = it->second.launches;
    L->profiled_last = L->profiling;
    L->last_xn = (T > qrm::route_small_max_tokens(L->desc.d_model) && !(flags & QRM_APPLY_NORM)) ? x : L->xn;
    return QRM_OK;
}

extern "C" int qrm_forward_device(qrm_layer* L, const float* x_dev, int T, int flags, float* out_dev,
                                  int32_t* topk_idx_dev, float* topk_w_dev, void* stream) {
    if (!L || !x_dev || !out_dev) return fail(QRM_E_INVALID, "NULL argument");
    int rc = forward_checks(L, T, flags);
    if (rc) return rc;
    QRM_CUDA(cudaSetDevice(L->desc.device));
    cudaStream_t s = stream ? (cudaStream_t)stream : L->stream;
    return run_forward(L, x_dev, T, flags, out_dev, topk_idx_dev ? topk_idx_dev : L->topk_idx,
                       topk_w_dev ? topk_w_dev : L->topk_w, s);
}

extern "C" int qrm_sync(qrm_layer* L) {
    if (!L) return fail(QRM_E_INVALID, "NULL layer");
    QRM_CUDA(cudaSetDevice(L->desc.device));
    QRM_CUDA(cudaDeviceSynchronize());
    int32_t err = 0;
    QRM_CUDA(cudaMemcpy(&err, &L->sched->err, sizeof(int32_t), cudaMemcpyDeviceToHost));
    if (err) {
        QRM_CUDA(cudaMemset(&L->sched->err, 0, sizeof(int32_t)));
        if (err & qrm::ERR_TIMEOUT) return fail(QRM_E_TIMEOUT, "a device wait timed out");
        return fail(QRM_E_INVALID, "device reported error flags 0x%x (expert index out of range)", err);
    }
    return QRM_OK;
}

// Batches whose rows fit this many bytes go through qrm_forward's pinned,
// mapped staging: the caller's inputs are copied on the host and uploaded by
// one asynchronous DMA, the combine writes the output rows, the top-k and the
// error flags straight into the mapped staging (no read-back DMA), and the
// call waits once (C5 decode: 176 -> 135 us per call).  A
// pageable transfer is staged by the driver on its own, and each pageable
// read-back and the separate error check wait for the device again (~78 us
// per call at C5 decode).  Above this size the two host copies cost more than
// the driver's pipelined pageable transfers.
constexpr size_t kHostStageBytes = 256u << 10;

static int forward_staged(qrm_layer* L, const float* x, int T, int flags, float* out, int32_t* topk_idx,
                          float* topk_w) {
    const int d = L->desc.d_model, k = L->k;
    const size_t xb = sizeof(float) * (size_t)T * d, kb = sizeof(int32_t) * (size_t)T * k;
    if (L->host_stage_rows < T) {
        const int rows = (int)std::max<size_t>((size_t)T, kHostStageBytes / (sizeof(float) * d));
        if (L->host_stage) cudaFreeHost(L->host_stage);
        L->host_stage = nullptr;
        L->host_stage_rows = 0;
        const size_t bytes = 2 * sizeof(float) * (size_t)rows * d + 2 * sizeof(int32_t) * (size_t)rows * k + 64;
        if (cudaHostAlloc(&L->host_stage, bytes, cudaHostAllocMapped) != cudaSuccess) {
            L->host_stage = nullptr;
            return fail(QRM_E_NOMEM, "pinned staging of %zu bytes", bytes);
        }
        L->host_stage_rows = rows;
    }
    const int cap = L->host_stage_rows;
    float* hx = reinterpret_cast<float*>(L->host_stage);
    float* hout = hx + (size_t)cap * d;
    int32_t* hidx = reinterpret_cast<int32_t*>(hout + (size_t)cap * d);
    float* hw = reinterpret_cast<float*>(hidx + (size_t)cap * k);
    int32_t* herr = reinterpret_cast<int32_t*>(hw + (size_t)cap * k);
    // device views of the mapped staging: the combine writes the output rows,
    // the top-k and the error flags there (a graph of this path always has
    // these pointers: its output pointer is the staging's own)
    float* dout = nullptr;
    QRM_CUDA(cudaHostGetDevicePointer(reinterpret_cast<void**>(&dout), hout, 0));
    QRM_CUDA(cudaHostGetDevicePointer(reinterpret_cast<void**>(&L->stage_idx), hidx, 0));
    QRM_CUDA(cudaHostGetDevicePointer(reinterpret_cast<void**>(&L->stage_w), hw, 0));
    QRM_CUDA(cudaHostGetDevicePointer(reinterpret_cast<void**>(&L->stage_err), herr, 0));
    *herr = -1;   // overwritten by the combine
    memcpy(hx, x, xb);
    QRM_CUDA(cudaMemcpyAsync(L->x, hx, xb, cudaMemcpyHostToDevice, L->stream));
    int rc = run_forward(L, L->x, T, flags, dout, L->topk_idx, L->topk_w, L->stream);
    L->stage_idx = nullptr;
    L->stage_w = nullptr;
    L->stage_err = nullptr;
    if (rc) return rc;
    QRM_CUDA(cudaStreamSynchronize(L->stream));
    const int32_t err = *reinterpret_cast<volatile int32_t*>(herr);
    if (err == -1) return fail(QRM_E_CUDA, "internal: the staged forward did not report its flags");
    if (err) {
        QRM_CUDA(cudaMemsetAsync(&L->sched->err, 0, sizeof(int32_t), L->stream));
        QRM_CUDA(cudaStreamSynchronize(L->stream));
        if (err & qrm::ERR_TIMEOUT) return fail(QRM_E_TIMEOUT, "a device wait timed out");
        return fail(QRM_E_INVALID, "device reported error flags 0x%x (expert index out of range)", err);
    }
    memcpy(out, hout, xb);
    if (topk_idx) memcpy(topk_idx, hidx, kb);
    if (topk_w) memcpy(topk_w, hw, kb);
    return QRM_OK;
}

extern "C" int qrm_forward(qrm_layer* L, const float* x, int T, int flags, float* out, int32_t* topk_idx, float* topk_w) {
    if (!L || !x || !out) return fail(QRM_E_INVALID, "NULL argument");
    int rc = forward_checks(L, T, flags);
    if (rc) return rc;
    QRM_CUDA(cudaSetDevice(L->desc.device));
    const size_t xb = sizeof(float) * (size_t)T * L->desc.d_model;
    // one process per GPU and one layer stream: the staged path covers
    // single-GPU layers; expert-parallel layers synchronise the whole device
    if (L->world == 1 && xb <= kHostStageBytes) return forward_staged(L, x, T, flags, out, topk_idx, topk_w);
    QRM_CUDA(cudaMemcpyAsync(L->x, x, xb, cudaMemcpyHostToDevice, L->stream));
    rc = run_forward(L, L->x, T, flags, L->out, L->topk_idx, L->topk_w, L->stream);
    if (rc) return rc;
    QRM_CUDA(cudaMemcpyAsync(out, L->out, xb, cudaMemcpyDeviceToHost, L->stream));
    if (topk_idx) QRM_CUDA(cudaMemcpyAsync(topk_idx, L->topk_idx, sizeof(int32_t) * T * L->k, cudaMemcpyDeviceToHost, L->stream));
    if (topk_w) QRM_CUDA(cudaMemcpyAsync(topk_w, L->topk_w, sizeof(float) * T * L->k, cudaMemcpyDeviceToHost, L->stream));
    QRM_CUDA(cudaStreamSynchronize(L->stream));
    return qrm_sync(L);
}

extern "C" int qrm_last_dispatch(qrm_layer* L, int32_t* perm, int32_t* offsets) {
    if (!L) return fail(QRM_E_INVALID, "NULL layer");
    if (!L->last_T) return fail(QRM_E_STATE, "no forward has run");
    QRM_CUDA(cudaSetDevice(L->desc.device));
    QRM_CUDA(cudaDeviceSynchronize());
    if (perm) QRM_CUDA(cudaMemcpy(perm, L->perm, sizeof(int32_t) * L->last_T * L->k, cudaMemcpyDeviceToHost));
    if (offsets) QRM_CUDA(cudaMemcpy(offsets, L->offsets, sizeof(int32_t) * (L->desc.n_experts + 1), cudaMemcpyDeviceToHost));
    return QRM_OK;
}

extern "C" int qrm_last_launch_count(qrm_layer* L, int* count) {
    if (!L || !count) return fail(QRM_E_INVALID, "NULL argument");
    if (L->last_T <= 0) return fail(QRM_E_STATE, "no forward has run");
    *count = L->last_launches;
    return QRM_OK;
}

extern "C" int qrm_last_router(qrm_layer* L, float* logits, float* xn) {
    if (!L) return fail(QRM_E_INVALID, "NULL layer");
    if (!L->last_T) return fail(QRM_E_STATE, "no forward has run");
    QRM_CUDA(cudaSetDevice(L->desc.device));
    QRM_CUDA(cudaDeviceSynchronize());
    if (logits) QRM_CUDA(cudaMemcpy(logits, L->logits, sizeof(float) * L->last_T * L->desc.n_experts, cudaMemcpyDeviceToHost));
    if (xn) QRM_CUDA(cudaMemcpy(xn, L->last_xn, sizeof(float) * L->last_T * L->desc.d_model, cudaMemcpyDeviceToHost));
    return QRM_OK;
}

extern "C" int qrm_set_profiling(qrm_layer* L, int on) {
    if (!L) return fail(QRM_E_INVALID, "NULL layer");
    QRM_CUDA(cudaSetDevice(L->desc.device));
    if (on && !L->ev[0])
        for (cudaEvent_t& e : L->ev) QRM_CUDA(cudaEventCreate(&e));
    L->profiling = on != 0;
    return QRM_OK;
}

extern "C" int qrm_last_profile_ep(qrm_layer* L, float* ms) {
    if (!L || !ms) return fail(QRM_E_INVALID, "NULL argument");
    if (L->world < 2) return fail(QRM_E_STATE, "not an expert-parallel layer (use qrm_last_profile)");
    if (!L->last_T || !L->profiled_last) return fail(QRM_E_STATE, "the last forward ran without profiling");
    QRM_CUDA(cudaSetDevice(L->desc.device));
    QRM_CUDA(cudaEventSynchronize(L->ev[QRM_EP_STAGE_COUNT]));
    for (int i = 0; i < QRM_EP_STAGE_COUNT; i++) QRM_CUDA(cudaEventElapsedTime(&ms[i], L->ev[i], L->ev[i + 1]));
    return QRM_OK;
}

extern "C" int qrm_last_profile(qrm_layer* L, float* ms, double* bytes) {
    if (!L) return fail(QRM_E_INVALID, "NULL layer");
    if (L->world > 1) return fail(QRM_E_STATE, "expert-parallel layer: use qrm_last_profile_ep");
    if (!L->last_T || !L->profiled_last) return fail(QRM_E_STATE, "the last forward ran without profiling");
    QRM_CUDA(cudaSetDevice(L->desc.device));
    QRM_CUDA(cudaEventSynchronize(L->ev[QRM_STAGE_COUNT]));
    if (ms)
        for (int i = 0; i < QRM_STAGE_COUNT; i++) QRM_CUDA(cudaEventElapsedTime(&ms[i], L->ev[i], L->ev[i + 1]));
    if (bytes) {
        int32_t na = 0;
        QRM_CUDA(cudaMemcpy(&na, &L->sched->n_active, sizeof na, cudaMemcpyDeviceToHost));
        const int E = L->desc.n_experts, T = L->last_T, k = L->k;
        const double d = L->desc.d_model, f = L->desc.expert_ffn;
        const size_t e0 = (size_t)L->first_expert * 3;
        double gu = (double)na * (L->mat_bytes[e0] + L->mat_bytes[e0 + 1]);
        double dn = (double)na * L->mat_bytes[e0 + 2];
        int tok_sh = L->last_shared ? T : 0;
        if (L->last_shared) {
            gu += (double)L->mat_bytes[(size_t)E * 3] + L->mat_bytes[(size_t)E * 3 + 1];
            dn += (double)L->mat_bytes[(size_t)E * 3 + 2];
        }
        // activations: xn read once, h written / read once, y written once
        gu += 4.0 * (T * d + ((double)T * k + tok_sh) * f);
        dn += 4.0 * (((double)T * k + tok_sh) * f + ((double)T * k + tok_sh) * d);
        for (int i = 0; i < QRM_STAGE_COUNT; i++) bytes[i] = 0;
        bytes[QRM_STAGE_GATEUP] = gu;
        bytes[QRM_STAGE_DOWN] = dn;
    }
    return QRM_OK;
}

// ---------------------------------------------------------------- layer stack
// n MoE layers of one shape run back to back on a device-resident residual
// stream (the MoE part of ForwardLegacy, StreamingEngine.cs:213-286: every
// layer x += MoeFfn(RmsNorm(x))).  The first n_res layers keep their weights
// in HBM; when the budget does not hold them all, the others keep theirs in
// pinned host images (the slab bytes in device layout, captured at upload)
// and are streamed through two device slots by layer parity, each copy on a
// copy stream overlapping the compute of the layer before -- the GPU
// counterpart of PrefetchPipeline's ping-pong staging (PrefetchPipeline.cs:
// 64-166), whose over-budget fallback (:131-135) becomes "stream from host".
struct qrm_stack {
    qrm_layer_desc desc{};
    int n = 0, n_res = 0;
    std::vector<qrm_layer*> layers;
    size_t slab_bytes = 0;
    uint8_t* slot[2] = {};
    std::vector<uint8_t*> images;      // [n - n_res] pinned host images
    cudaStream_t copy = nullptr;
    cudaEvent_t copied[2] = {}, freed[2] = {};
    float* act[2] = {};                // residual stream between layers [max_tokens][d]
};

static void free_stack(qrm_stack* S) {
    if (!S) return;
    cudaSetDevice(S->desc.device);
    cudaDeviceSynchronize();
    for (qrm_layer* L : S->layers) free_layer(L);
    for (uint8_t* p : S->images)
        if (p) cudaFreeHost(p);
    for (int i = 0; i < 2; i++) {
        if (S->slot[i]) cudaFree(S->slot[i]);
        if (S->act[i]) cudaFree(S->act[i]);
        if (S->copied[i]) cudaEventDestroy(S->copied[i]);
        if (S->freed[i]) cudaEventDestroy(S->freed[i]);
    }
    if (S->copy) cudaStreamDestroy(S->copy);
    delete S;
}

extern "C" int qrm_stack_create(const qrm_layer_desc* desc, int n_layers, size_t hbm_budget, qrm_stack** out) {
    if (!out) return fail(QRM_E_INVALID, "out is NULL");
    *out = nullptr;
    int rc = check_desc(desc);
    if (rc) return rc;
    if (n_layers <= 0) return fail(QRM_E_INVALID, "n_layers must be positive");
    QRM_CUDA(cudaSetDevice(desc->device));
    qrm_stack* S = new qrm_stack();
    S->desc = *desc;
    S->n = n_layers;
    auto bail = [&](int code) { free_stack(S); return code; };
    // layer 0 tells the slab size of every layer (one shape)
    qrm_layer* L0 = nullptr;
    if ((rc = create_layer(desc, 0, 1, nullptr, &L0))) return bail(rc);
    S->layers.push_back(L0);
    S->slab_bytes = L0->slab_bytes;
    const size_t lb = S->slab_bytes;
    if (hbm_budget == 0 || lb * (size_t)n_layers <= hbm_budget) {
        S->n_res = n_layers;
    } else {
        // two slots for the streamed layers, the rest of the budget resident
        S->n_res = hbm_budget >= 2 * lb ? (int)std::min<size_t>((hbm_budget - 2 * lb) / lb, n_layers) : 0;
        S->n_res = std::max(S->n_res, 1);   // layer 0 exists already
        if (S->n_res >= n_layers) S->n_res = n_layers;
    }
    const int ns = n_layers - S->n_res;
    if (ns > 0) {
        if (cudaMalloc(&S->slot[0], lb) != cudaSuccess || cudaMalloc(&S->slot[1], lb) != cudaSuccess)
            return bail(fail(QRM_E_NOMEM, "stream slots (2 x %zu bytes)", lb));
        if (cudaStreamCreateWithFlags(&S->copy, cudaStreamNonBlocking) != cudaSuccess)
            return bail(fail(QRM_E_CUDA, "copy stream"));
        for (int i = 0; i < 2; i++) {
            if (cudaEventCreateWithFlags(&S->copied[i], cudaEventDisableTiming) != cudaSuccess ||
                cudaEventCreateWithFlags(&S->freed[i], cudaEventDisableTiming) != cudaSuccess)
                return bail(fail(QRM_E_CUDA, "events"));
            QRM_CUDA(cudaEventRecord(S->freed[i], S->copy));
        }
    }
    for (int l = 1; l < n_layers; l++) {
        qrm_layer* L = nullptr;
        const bool streamed = l >= S->n_res;
        if ((rc = create_layer(desc, 0, 1, nullptr, &L, streamed ? S->slot[(l - S->n_res) & 1] : nullptr)))
            return bail(rc);
        S->layers.push_back(L);
        if (streamed) {
            uint8_t* img = nullptr;
            if (cudaMallocHost(&img, lb) != cudaSuccess)
                return bail(fail(QRM_E_NOMEM, "pinned host image of layer %d (%zu bytes)", l, lb));
            memset(img, 0, lb);
            S->images.push_back(img);
            L->image = img;
        }
    }
    for (int i = 0; i < 2; i++)
        if (cudaMalloc(&S->act[i], sizeof(float) * (size_t)desc->max_tokens * desc->d_model) != cudaSuccess)
            return bail(fail(QRM_E_NOMEM, "residual stream buffers"));
    *out = S;
    return QRM_OK;
}

extern "C" void qrm_stack_destroy(qrm_stack* S) { free_stack(S); }

extern "C" int qrm_stack_layer(qrm_stack* S, int i, qrm_layer** layer) {
    if (!S || !layer) return fail(QRM_E_INVALID, "NULL argument");
    if (i < 0 || i >= S->n) return fail(QRM_E_INVALID, "layer %d of %d", i, S->n);
    *layer = S->layers[i];
    return QRM_OK;
}

extern "C" int qrm_stack_info(qrm_stack* S, int* n_resident, size_t* layer_bytes) {
    if (!S) return fail(QRM_E_INVALID, "NULL stack");
    if (n_resident) *n_resident = S->n_res;
    if (layer_bytes) *layer_bytes = S->slab_bytes;
    return QRM_OK;
}

extern "C" int qrm_stack_load_qw(qrm_stack* S, const char* path, int first_layer) {
    if (!S) return fail(QRM_E_INVALID, "NULL stack");
    for (int l = 0; l < S->n; l++) {
        int rc = qrm_load_qw(S->layers[l], path, first_layer + l);
        if (rc) return rc;
    }
    return QRM_OK;
}

extern "C" int qrm_stack_forward_device(qrm_stack* S, const float* x_dev, int T, int flags, float* out_dev,
                                        void* stream) {
    if (!S || !x_dev || !out_dev) return fail(QRM_E_INVALID, "NULL argument");
    if (T <= 0 || T > S->desc.max_tokens) return fail(QRM_E_CAPACITY, "T = %d outside 1..%d", T, S->desc.max_tokens);
    QRM_CUDA(cudaSetDevice(S->desc.device));
    cudaStream_t s = stream ? (cudaStream_t)stream : S->layers[0]->stream;
    const int ns = S->n - S->n_res;
    // the first two streamed layers' weights go into their slots as soon as
    // the layers that used the slots in the previous forward are done
    auto issue = [&](int j) -> int {   // streamed layer j (layer n_res + j) into slot j & 1
        const int sl = j & 1;
        QRM_CUDA(cudaStreamWaitEvent(S->copy, S->freed[sl], 0));
        QRM_CUDA(cudaMemcpyAsync(S->slot[sl], S->images[j], S->slab_bytes, cudaMemcpyHostToDevice, S->copy));
        QRM_CUDA(cudaEventRecord(S->copied[sl], S->copy));
        return QRM_OK;
    };
    int rc;
    for (int j = 0; j < std::min(ns, 2); j++)
        if ((rc = issue(j))) return rc;
    const float* cur = x_dev;
    for (int l = 0; l < S->n; l++) {
        float* dst = l == S->n - 1 ? out_dev : S->act[l & 1];
        const int j = l - S->n_res;
        if (j >= 0) QRM_CUDA(cudaStreamWaitEvent(s, S->copied[j & 1], 0));
        rc = qrm_forward_device(S->layers[l], cur, T, flags, dst, nullptr, nullptr, s);
        if (rc) return rc;
        if (j >= 0) {
            QRM_CUDA(cudaEventRecord(S->freed[j & 1], s));
            if (j + 2 < ns && (rc = issue(j + 2))) return rc;
        }
        cur = dst;
    }
    return QRM_OK;
}

extern "C" int qrm_stack_sync(qrm_stack* S) {
    if (!S) return fail(QRM_E_INVALID, "NULL stack");
    for (qrm_layer* L : S->layers) {
        int rc = qrm_sync(L);
        if (rc) return rc;
    }
    return QRM_OK;
}

// ---------------------------------------------------------------- matrix operator

struct qrm_matrix {
    int device = 0;
    int sm_count = 0;
    int64_t bytes = 0;
    qrm::MatDev mat{};
    qrm::MatDev* mats_dev = nullptr;  // [3]; slot 2 is the matrix
    uint8_t* data = nullptr;
    int32_t* misc = nullptr;          // active[1], offsets[2], n_active, ctr, err
    uint8_t* xtab = nullptr;          // activation tables of the last call's rows
    int xtab_rows = 0;
};

extern "C" int qrm_matrix_create(int device, int fmt, int64_t rows, int64_t cols, const void* bytes, size_t nbytes,
                                 qrm_matrix** out) {
    if (!out || !bytes) return fail(QRM_E_INVALID, "NULL argument");
    *out = nullptr;
    if (!qrm::is_expert_fmt(fmt)) return fail(QRM_E_FORMAT, "format %d has no GPU kernel", fmt);
    if (rows <= 0 || cols <= 0 || cols % 32 || cols / 32 > qrm::kGemvMaxThreads || rows > (1 << 30))
        return fail(QRM_E_INVALID, "unsupported shape %lld x %lld", (long long)rows, (long long)cols);
    int64_t nb = tensor_bytes(fmt, rows, cols);
    if (nb < 0) return fail(QRM_E_INVALID, "cols %lld not a multiple of the block size", (long long)cols);
    if ((size_t)nb != nbytes) return fail(QRM_E_SIZE, "%zu bytes, TensorBytes = %lld", nbytes, (long long)nb);
    cudaDeviceProp prop;
    QRM_CUDA(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10) return fail(QRM_E_CUDA, "device %d is not sm_100", device);
    QRM_CUDA(cudaSetDevice(device));
    qrm_matrix* M = new qrm_matrix();
    M->device = device;
    M->sm_count = prop.multiProcessorCount;
    M->bytes = nb;
    auto bail = [&](int code) {
        if (M->data) cudaFree(M->data);
        if (M->mats_dev) cudaFree(M->mats_dev);
        if (M->misc) cudaFree(M->misc);
        delete M;
        return code;
    };
    uint8_t* staging = nullptr;
    if (cudaMalloc(&M->data, nbytes) != cudaSuccess || cudaMalloc(&staging, nbytes) != cudaSuccess)
        return bail(fail(QRM_E_NOMEM, "matrix allocation failed"));
    cudaMemcpy(staging, bytes, nbytes, cudaMemcpyHostToDevice);
    int bs, bb;
    qrm::block_spec(fmt, &bs, &bb);
    if (imma_usable(fmt, (int)rows, (int)cols, false))
        qrm::tile_relayout_kernel<<<M->sm_count * 8, 256>>>(fmt, bb, (int)(cols / 256), staging, M->data,
                                                            (long long)(nbytes / bb), 1);
    else if (fmt == qrm::Q4_K || qrm::is_raw_fmt(fmt)) cudaMemcpy(M->data, staging, nbytes, cudaMemcpyDeviceToDevice);
    else qrm::relayout_kernel<<<M->sm_count * 8, 256>>>(fmt, bb, staging, M->data, (long long)(nbytes / bb), 1);
    cudaError_t e = cudaDeviceSynchronize();
    cudaFree(staging);
    if (e != cudaSuccess) return bail(fail(QRM_E_CUDA, "matrix upload: %s", cudaGetErrorString(e)));
    M->mat = qrm::MatDev{M->data, fmt, (int32_t)rows, (int32_t)cols, 0, rows * cols / bs};
    qrm::MatDev tab[3] = {M->mat, M->mat, M->mat};
    int32_t misc[8] = {0, 0, 0, 0, 0, 0, 0, 0};  // active[0]=0, offsets, n_active=0, ctr
    if (cudaMalloc(&M->mats_dev, sizeof tab) != cudaSuccess || cudaMalloc(&M->misc, sizeof misc) != cudaSuccess)
        return bail(fail(QRM_E_NOMEM, "matrix table allocation failed"));
    cudaMemcpy(M->mats_dev, tab, sizeof tab, cudaMemcpyHostToDevice);
    cudaMemcpy(M->misc, misc, sizeof misc, cudaMemcpyHostToDevice);
    *out = M;
    return QRM_OK;
}

extern "C" void qrm_matrix_destroy(qrm_matrix* M) {
    if (!M) return;
    cudaSetDevice(M->device);
    cudaDeviceSynchronize();
    if (M->data) cudaFree(M->data);
    if (M->mats_dev) cudaFree(M->mats_dev);
    if (M->misc) cudaFree(M->misc);
    if (M->xtab) cudaFree(M->xtab);
    delete M;
}

extern "C" int qrm_matrix_gemv(qrm_matrix* M, const float* x_dev, int T, float* y_dev, void* stream) {
    if (!M || !x_dev || !y_dev) return fail(QRM_E_INVALID, "NULL argument");
    if (T <= 0) return fail(QRM_E_INVALID, "T must be positive");
    QRM_CUDA(cudaSetDevice(M->device));
    cudaStream_t s = (cudaStream_t)stream;
    // the matrix runs as the "shared expert" slot of a one-expert layer
    QRM_CUDA(cudaMemsetAsync(M->misc + 4, 0, sizeof(int32_t), s));
    qrm::GemvParams gp{};
    gp.mats = M->mats_dev;
    gp.active = M->misc;        // active[0] = 0
    gp.offsets = M->misc + 1;
    gp.perm = M->misc;
    gp.n_active = M->misc + 3;  // 0 routed slots
    gp.ctr = M->misc + 4;
    gp.x_routed = x_dev;
    gp.x_shared = x_dev;
    gp.out_routed = y_dev;
    gp.out_shared = y_dev;
    gp.T = T;
    gp.T_sh = T;
    gp.k = 1;
    gp.E = 0;
    gp.rows = M->mat.rows;
    gp.cols = M->mat.cols;
    gp.tiles = (gp.rows + kRDown - 1) / kRDown;
    gp.limit = 0.f;
    gp.routed_by_token = 0;
    gp.mode = 2;
    gp.has_shared = 1;
    if (imma_usable(M->mat.fmt, M->mat.rows, M->mat.cols, false)) {
        if (M->xtab_rows < T) {
            QRM_CUDA(cudaStreamSynchronize(s));
            if (M->xtab) cudaFree(M->xtab);
            M->xtab = nullptr;
            M->xtab_rows = 0;
            if (cudaMalloc(&M->xtab, (size_t)qrm::xtab_stride(M->mat.cols) * T) != cudaSuccess)
                return fail(QRM_E_NOMEM, "activation table allocation failed");
            M->xtab_rows = T;
        }
        int rc = launch_xquant(x_dev, M->mat.cols, T, M->xtab, s);
        if (rc) return rc;
        gp.xtab = M->xtab;
        gp.xtab_stride = qrm::xtab_stride(M->mat.cols);
        gp.xtab_shared_base = 0;
        gp.xtab_rows = T;
    }
    return launch_gemv(M->mat.fmt, false, pick_nt(T), gp, M->sm_count, M->misc + 5, s);
}

// ---------------------------------------------------------------- dense FFN
// StreamingEngine.DenseFfn / DenseFfnOut (StreamingEngine.cs:599-622) from
// three matrix operators: g = W_gate xn, u = W_up xn, h = SwiGLU(g, u),
// y = W_down h, out = x + y (AxpyF32 with alpha 1) or out = y.
struct qrm_ffn {
    qrm_matrix* m[3] = {};
    int device = 0, d = 0, f = 0, max_tokens = 0, sm_count = 0;
    float *g = nullptr, *u = nullptr, *y = nullptr;
};

namespace qrm {
// h = SwiGLU(g, u) in place of g (Glm5Ops.LimitedSwiglu / SiluMulInPlace)
__global__ void ffn_swiglu_kernel(float* __restrict__ g, const float* __restrict__ u, long long n, float limit) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        g[i] = swiglu(g[i], u[i], limit);
}
// out = x + 1 * y (SimdMath.AxpyF32, alpha 1: the product is exact) or y
__global__ void ffn_residual_kernel(const float* __restrict__ x, const float* __restrict__ y, float* __restrict__ out,
                                    long long n) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        out[i] = x ? __fadd_rn(x[i], y[i]) : y[i];
}
}  // namespace qrm

extern "C" int qrm_ffn_create(qrm_matrix* gate, qrm_matrix* up, qrm_matrix* down, int max_tokens, qrm_ffn** out) {
    if (!out || !gate || !up || !down) return fail(QRM_E_INVALID, "NULL argument");
    *out = nullptr;
    if (max_tokens <= 0) return fail(QRM_E_INVALID, "max_tokens must be positive");
    if (gate->device != up->device || gate->device != down->device)
        return fail(QRM_E_INVALID, "the three matrices are on different devices");
    const int f = gate->mat.rows, d = gate->mat.cols;
    if (up->mat.rows != f || up->mat.cols != d || down->mat.rows != d || down->mat.cols != f)
        return fail(QRM_E_INVALID, "shapes gate %dx%d, up %dx%d, down %dx%d do not form an FFN", gate->mat.rows,
                    gate->mat.cols, up->mat.rows, up->mat.cols, down->mat.rows, down->mat.cols);
    QRM_CUDA(cudaSetDevice(gate->device));
    qrm_ffn* F = new qrm_ffn();
    F->m[0] = gate;
    F->m[1] = up;
    F->m[2] = down;
    F->device = gate->device;
    F->d = d;
    F->f = f;
    F->max_tokens = max_tokens;
    F->sm_count = gate->sm_count;
    if (cudaMalloc(&F->g, sizeof(float) * (size_t)max_tokens * f) != cudaSuccess ||
        cudaMalloc(&F->u, sizeof(float) * (size_t)max_tokens * f) != cudaSuccess ||
        cudaMalloc(&F->y, sizeof(float) * (size_t)max_tokens * d) != cudaSuccess) {
        if (F->g) cudaFree(F->g);
        if (F->u) cudaFree(F->u);
        delete F;
        return fail(QRM_E_NOMEM, "FFN work buffers");
    }
    *out = F;
    return QRM_OK;
}

extern "C" void qrm_ffn_destroy(qrm_ffn* F) {
    if (!F) return;
    cudaSetDevice(F->device);
    cudaDeviceSynchronize();
    cudaFree(F->g);
    cudaFree(F->u);
    cudaFree(F->y);
    delete F;
}

extern "C" int qrm_ffn_forward(qrm_ffn* F, const float* xn_dev, const float* x_dev, int T, float swiglu_limit,
                               float* out_dev, void* stream) {
    if (!F || !xn_dev || !out_dev) return fail(QRM_E_INVALID, "NULL argument");
    if (T <= 0 || T > F->max_tokens) return fail(QRM_E_CAPACITY, "T = %d outside 1..%d", T, F->max_tokens);
    QRM_CUDA(cudaSetDevice(F->device));
    cudaStream_t s = (cudaStream_t)stream;
    int rc;
    if ((rc = qrm_matrix_gemv(F->m[0], xn_dev, T, F->g, stream))) return rc;
    if ((rc = qrm_matrix_gemv(F->m[1], xn_dev, T, F->u, stream))) return rc;
    const long long nf = (long long)T * F->f, nd = (long long)T * F->d;
    qrm::ffn_swiglu_kernel<<<(int)std::min<long long>((nf + 255) / 256, (long long)F->sm_count * 8), 256, 0, s>>>(
        F->g, F->u, nf, swiglu_limit);
    QRM_CUDA(cudaGetLastError());
    if ((rc = qrm_matrix_gemv(F->m[2], F->g, T, F->y, stream))) return rc;
    qrm::ffn_residual_kernel<<<(int)std::min<long long>((nd + 255) / 256, (long long)F->sm_count * 8), 256, 0, s>>>(
        x_dev, F->y, out_dev, nd);
    QRM_CUDA(cudaGetLastError());
    return QRM_OK;
}

// ---------------------------------------------------------------- matrix operator, no allocation
// qrm_matrix_gemv_static keeps the activation tables of the integer
// tensor-core kernel in this fixed device array (one copy per device, shared
// by every call on that device) instead of the matrix's growable buffer.  The
// tables need no zeroing: xquant_kernel writes every byte the GEMV reads.
constexpr size_t kStaticTabBytes = (size_t)1 << 20;
static __device__ __align__(256) uint8_t g_static_tab[kStaticTabBytes];

namespace {
constexpr int kStaticMaxDevices = 64;
std::mutex g_static_mu;
uint8_t* g_static_tab_ptr[kStaticMaxDevices];  // device address of g_static_tab, per device
}  // namespace

extern "C" int qrm_matrix_gemv_static(qrm_matrix* M, const float* x_dev, int T, float* y_dev, void* stream) {
    if (!M || !x_dev || !y_dev) return fail(QRM_E_INVALID, "NULL argument");
    if (T <= 0) return fail(QRM_E_INVALID, "T must be positive");
    if (M->device < 0 || M->device >= kStaticMaxDevices)
        return fail(QRM_E_INVALID, "device %d is outside the static scratch table", M->device);
    QRM_CUDA(cudaSetDevice(M->device));
    cudaStream_t s = (cudaStream_t)stream;
    const bool tables = imma_usable(M->mat.fmt, M->mat.rows, M->mat.cols, false);
    uint8_t* tab = nullptr;
    if (tables) {
        const size_t need = (size_t)qrm::xtab_stride(M->mat.cols) * (size_t)T;
        if (need > kStaticTabBytes)
            return fail(QRM_E_CAPACITY, "T = %d needs %zu bytes of activation tables; the static scratch holds %zu",
                        T, need, kStaticTabBytes);
        std::lock_guard<std::mutex> lock(g_static_mu);
        if (!g_static_tab_ptr[M->device]) {
            void* p = nullptr;
            cudaError_t e = cudaGetSymbolAddress(&p, g_static_tab);
            if (e != cudaSuccess) return fail(QRM_E_CUDA, "static scratch address: %s", cudaGetErrorString(e));
            g_static_tab_ptr[M->device] = static_cast<uint8_t*>(p);
        }
        tab = g_static_tab_ptr[M->device];
    }
    QRM_CUDA(cudaMemsetAsync(M->misc + 4, 0, sizeof(int32_t), s));
    qrm::GemvParams gp{};
    gp.mats = M->mats_dev;
    gp.active = M->misc;
    gp.offsets = M->misc + 1;
    gp.perm = M->misc;
    gp.n_active = M->misc + 3;
    gp.ctr = M->misc + 4;
    gp.x_routed = x_dev;
    gp.x_shared = x_dev;
    gp.out_routed = y_dev;
    gp.out_shared = y_dev;
    gp.T = T;
    gp.T_sh = T;
    gp.k = 1;
    gp.E = 0;
    gp.rows = M->mat.rows;
    gp.cols = M->mat.cols;
    gp.tiles = (gp.rows + kRDown - 1) / kRDown;
    gp.limit = 0.f;
    gp.routed_by_token = 0;
    gp.mode = 2;
    gp.has_shared = 1;
    if (tables) {
        int rc = launch_xquant(x_dev, M->mat.cols, T, tab, s);
        if (rc) return rc;
        gp.xtab = tab;
        gp.xtab_stride = qrm::xtab_stride(M->mat.cols);
        gp.xtab_shared_base = 0;
        gp.xtab_rows = T;
    }
    return launch_gemv(M->mat.fmt, false, pick_nt(T), gp, M->sm_count, M->misc + 5, s);
}

// ---------------------------------------------------------------- self-tests
namespace qrm {
// the binary32 exp of the routing kernels on consecutive bit patterns
__global__ void selftest_expf_kernel(uint32_t first, uint32_t count, uint32_t* __restrict__ out) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < count; i += gridDim.x * blockDim.x)
        out[i] = __float_as_uint(expf_glibc(__uint_as_float(first + i)));
}
// the library's give-up waits on things nothing completes: warp 0 on an
// mbarrier nothing arrives at (the expert kernels' stage wait), warp 1 on a
// peer flag nothing raises (the expert-parallel wait); each records whether
// it gave up
__global__ void selftest_waits_kernel(const uint32_t* flag, int32_t* err, int32_t* gave_up) {
    __shared__ uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        abort_flag = 0;
        fence_barrier_init();
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warp == 0) {
        const bool ok = mbar_wait_abort(&bar, 0u, &abort_flag);
        if (lane == 0) {
            gave_up[0] = ok ? 0 : 1;
            if (!ok) atomicOr(err, (int)ERR_TIMEOUT);
        }
    } else if (warp == 1 && lane == 0) {
        const bool ok = ep_wait_flag(flag, 1u);
        gave_up[1] = ok ? 0 : 1;
        if (!ok) atomicOr(err, (int)ERR_TIMEOUT);
    }
}
}  // namespace qrm

extern "C" int qrm_selftest_expf(uint32_t first, uint32_t count, uint32_t* out_dev, void* stream) {
    if (!out_dev) return fail(QRM_E_INVALID, "NULL argument");
    if (!count) return QRM_OK;
    qrm::selftest_expf_kernel<<<1184, 256, 0, (cudaStream_t)stream>>>(first, count, out_dev);
    QRM_CUDA(cudaGetLastError());
    return QRM_OK;
}

extern "C" int qrm_selftest_waits(int device, int64_t limit_us, int* gave_up) {
    if (limit_us <= 0 || limit_us > 10000000) return fail(QRM_E_INVALID, "limit %lld us outside 1 us .. 10 s", (long long)limit_us);
    QRM_CUDA(cudaSetDevice(device));
    int32_t* buf = nullptr;   // flag | err | gave_up[2]
    QRM_CUDA(cudaMalloc(&buf, 4 * sizeof(int32_t)));
    QRM_CUDA(cudaMemset(buf, 0, 4 * sizeof(int32_t)));
    uint64_t old = 0;
    cudaMemcpyFromSymbol(&old, qrm::g_wait_limit_ns, sizeof old);
    QRM_CUDA(qrm::set_wait_limit_here((uint64_t)limit_us * 1000ull));
    qrm::selftest_waits_kernel<<<1, 64>>>(reinterpret_cast<const uint32_t*>(buf), buf + 1, buf + 2);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    int32_t h[4] = {};
    if (e == cudaSuccess) e = cudaMemcpy(h, buf, sizeof h, cudaMemcpyDeviceToHost);
    qrm::set_wait_limit_here(old);
    cudaFree(buf);
    if (e != cudaSuccess) return fail(QRM_E_CUDA, "wait self-test: %s", cudaGetErrorString(e));
    if (gave_up) {
        gave_up[0] = h[2];
        gave_up[1] = h[3];
    }
    return (h[1] & qrm::ERR_TIMEOUT) ? fail(QRM_E_TIMEOUT, "bounded waits gave up after %lld us", (long long)limit_us)
                                     : QRM_OK;
}

// ---------------------------------------------------------------- synthetic data

extern "C" int qrm_synth_gaussian(float* dst_dev, int64_t n, uint64_t seed, float sigma, void* stream) {
    if (!dst_dev) return fail(QRM_E_INVALID, "NULL argument");
    int rc = qrm_synth_gaussian_impl(dst_dev, n, seed, sigma, (cudaStream_t)stream);
    return rc ? fail(rc, "synthetic Gaussian launch failed") : QRM_OK;
}

extern "C" int qrm_synth_quantize(int fmt, const float* src_dev, int64_t n, void* dst_dev, void* stream) {
    if (!src_dev || !dst_dev) return fail(QRM_E_INVALID, "NULL argument");
    int rc = qrm_synth_quantize_impl(fmt, src_dev, n, dst_dev, (cudaStream_t)stream);
    return rc ? fail(rc, "quantiser launch failed (format %d, n %lld)", fmt, (long long)n) : QRM_OK;
}
