/*
 * qrmoe.h -- C ABI of libqrmoe.so, the B200 (sm_100a) implementation of
 * QuantRunner's MoE FFN layer.
 *
 * The reference runs this layer on the CPU inside StreamingEngine (C#):
 *   MoeFfn         src/QuantRunner.Core/Runtime/StreamingEngine.cs:626-667
 *   LegacyMoeInto  StreamingEngine.cs:670-712
 *   GlmMoeFfn      StreamingEngine.cs:720-790
 * called from ForwardLegacy (StreamingEngine.cs:259-262) and ForwardGlm5
 * (StreamingEngine.cs:320-330), each expert product going through the public
 * operator DotKernels.MatVecParallel(QuantFormat, byte* w, long rows,
 * long cols, float* x, float* y) (src/QuantRunner.Core/Kernels/
 * DotKernels.cs:610).  A P/Invoke shim binds the entry points below so the
 * engine can hand a whole MoE layer to the GPU.
 *
 * Conventions: every function returns QRM_OK (0) or a negative QRM_E_* code;
 * qrm_last_error() then describes the failure (thread-local, valid until the
 * next call on the same thread).  Pointers named *_dev are device pointers of
 * the layer's device; all others are host pointers.  Calls on one qrm_layer
 * must not overlap (the reference engine is single-threaded too,
 * StreamingEngine.cs:39,103-117); distinct layers are independent.  There is
 * no CPU fallback: without a usable sm_100 device, qrm_create fails.
 */
#ifndef QRMOE_H
#define QRMOE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QRM_ABI_VERSION 1

/* Status codes.  The reference throws; the shim maps a negative code to
 * InvalidOperationException(qrm_last_error()). */
enum {
    QRM_OK = 0,
    QRM_E_INVALID = -1,   /* bad argument or shape  (ArgumentException, Dtypes.cs:63) */
    QRM_E_FORMAT = -2,    /* format id not supported (NotSupportedException, DotKernels.cs:44) */
    QRM_E_SIZE = -3,      /* byte count != Dtypes.TensorBytes (Dtypes.cs:60-65) */
    QRM_E_STATE = -4,     /* a tensor the forward needs was never uploaded (KeyNotFoundException, ModelStore.cs:79-80) */
    QRM_E_CUDA = -5,      /* CUDA runtime error */
    QRM_E_NCCL = -6,      /* NCCL error (expert-parallel layers) */
    QRM_E_TIMEOUT = -7,   /* a bounded device wait or a collective gave up */
    QRM_E_NOMEM = -8,     /* device allocation failed */
    QRM_E_CAPACITY = -9   /* request exceeds a fixed capacity */
};

/* QuantFormat ids as stored in .qw headers (src/QuantRunner.Core/Dtypes.cs:6-26).
 * Expert matrices may use any block format: Q4_0, Q8_0, Q4_K, Q6_K and TRI
 * run on the tensor-core kernels; Q2_K, Q3_K, Q5_K, I8_BLK, B1, B1X, T1E and
 * T1E_LO are kept exactly as stored and run on the CUDA-core kernel
 * (decoders of BlockDequantizer.cs, T1E's rANS stream of EntropyCoder.cs). */
enum {
    QRM_F32 = 0, QRM_F16 = 1, QRM_BF16 = 2, QRM_Q4_0 = 3, QRM_Q8_0 = 4, QRM_Q2_K = 5,
    QRM_Q4_K = 6, QRM_Q6_K = 7, QRM_TRI = 8, QRM_I8_BLK = 9, QRM_Q3_K = 10, QRM_Q5_K = 11,
    QRM_B1 = 12, QRM_B1X = 13, QRM_T1E = 14, QRM_T1E_LO = 15
};

/* Which matrix of an expert (canonical names, src/QuantRunner.Core/Models/
 * NameMapper.cs:7-12: l{i}.e{j}.w_gate / w_up / w_down, shared l{i}.sw_*). */
enum { QRM_GATE = 0, QRM_UP = 1, QRM_DOWN = 2 };
#define QRM_SHARED_EXPERT (-1)

/* Forward flags. */
enum {
    QRM_APPLY_NORM = 1,    /* input is the residual stream: xn = RmsNorm(x, ffn_norm) first
                              (StreamingEngine.cs:259-260 / 320-321) */
    QRM_ADD_RESIDUAL = 2   /* MoeFfn semantics: out = x + sum_j w_j y_j (StreamingEngine.cs:665);
                              without it out = sum_j w_j y_j (LegacyMoeInto / GlmMoeFfn) */
};

/* Layer description: the MoE fields of ModelConfig (src/QuantRunner.Core/
 * Models/ModelConfig.cs:22-61) plus storage formats and placement. */
typedef struct qrm_layer_desc {
    int32_t d_model;       /* "dim"          ModelConfig.cs:14 */
    int32_t n_experts;     /* "n_experts"    ModelConfig.cs:23 */
    int32_t n_active;      /* "n_active"     ModelConfig.cs:24 (top-k = min(n_active, 8), StreamingEngine.cs:628) */
    int32_t expert_ffn;    /* EffectiveExpertFfn ModelConfig.cs:25,67 (also the shared expert's width, StreamingEngine.cs:723,784) */
    int32_t moe_sigmoid;   /* "moe_sigmoid"  ModelConfig.cs:57: 1 = GlmMoeFfn routing */
    float   routed_scale;  /* "routed_scale" ModelConfig.cs:58 */
    int32_t n_shared;      /* "n_shared"     ModelConfig.cs:59 (GLM shared expert when > 0) */
    float   swiglu_limit;  /* "swiglu_limit" ModelConfig.cs:61 (GLM only; 0 = plain SiLU) */
    float   rms_eps;       /* "rms_eps"      ModelConfig.cs:22 */
    int32_t fmt_gate, fmt_up, fmt_down;          /* routed experts' storage formats */
    int32_t fmt_sh_gate, fmt_sh_up, fmt_sh_down; /* shared expert's storage formats */
    int32_t device;        /* CUDA device ordinal */
    int32_t max_tokens;    /* largest T per forward (buffers are sized for it) */
} qrm_layer_desc;

typedef struct qrm_layer qrm_layer;

/* ---- library ---- */
int         qrm_version(void);          /* QRM_ABI_VERSION */
const char* qrm_last_error(void);

/* ---- layer lifetime ----
 * qrm_create: replaces the per-layer state the engine reads through W()
 * (StreamingEngine.cs:186-192) and the PrefetchPipeline staging
 * (PrefetchPipeline.cs:64-166): the layer's experts live in HBM. */
int  qrm_create(const qrm_layer_desc* desc, qrm_layer** out);
void qrm_destroy(qrm_layer* layer);
/* The description the layer was created with. */
int  qrm_layer_get_desc(qrm_layer* layer, qrm_layer_desc* desc);

/* ---- uploads (host bytes are copied; the caller may unmap afterwards) ----
 * Replace Dequant1D(l{i}.ffn_norm) (StreamingEngine.cs:196-201,259),
 * Store.Get(l{i}.router) (:639) and l{i}.router_bias (:738-739), with the
 * tensors already widened to f32 (F16/BF16 widening is exact, Dtypes.cs:76-129). */
int qrm_upload_norm(qrm_layer* layer, const float* w /* [d] */);
int qrm_upload_router(qrm_layer* layer, const float* w /* [E x d] */, const float* bias /* [E] or NULL */);
/* Harness-only per-expert logit offset (added after the router dot; NULL
 * clears it).  No counterpart in the reference. */
int qrm_upload_logit_offset(qrm_layer* layer, const float* offset /* [E] or NULL */);
/* One expert matrix in its .qw block bytes (l{i}.e{j}.w_gate/w_up/w_down,
 * gate/up [f x d], down [d x f], row-major, blocks along columns,
 * ModelStore.cs:30-42).  expert = QRM_SHARED_EXPERT for l{i}.sw_*.  nbytes must
 * equal Dtypes.TensorBytes(rows*cols, fmt).  No requantisation: the bytes are
 * stored as they are, with each block's fields grouped by kind for aligned
 * loads (qrm_download_expert returns the original bytes). */
int qrm_upload_expert(qrm_layer* layer, int expert, int which, int fmt,
                      const void* bytes, size_t nbytes);
/* Same from device memory of the layer's device; the call synchronises the
 * device first, so bytes written by work on any stream are complete. */
int qrm_upload_expert_device(qrm_layer* layer, int expert, int which, int fmt,
                             const void* bytes_dev, size_t nbytes);
int qrm_download_expert(qrm_layer* layer, int expert, int which, void* bytes, size_t nbytes);

/* ---- .qw weight files (ModelStore.Open, src/QuantRunner.Core/Memory/
 * ModelStore.cs:85-126) ----
 * qrm_qw_layer_desc fills *out for MoE layer `layer_index` of the file: the
 * ModelConfig fields of the header's "config" (ModelConfig.cs:14-61; d_ff =
 * EffectiveExpertFfn), the formats of l{i}.e0.w_gate / w_up / w_down and of
 * l{i}.sw_* (n_shared becomes 0 when those tensors are absent, as the engine
 * skips the shared expert then, StreamingEngine.cs:779), plus the caller's
 * device and max_tokens.  No GPU work.  QRM_E_STATE when the layer has no
 * l{i}.router (a dense FFN layer, StreamingEngine.cs:633-637).
 * qrm_load_qw maps the file read-only for the call and uploads layer
 * `layer_index`'s tensors by their canonical names (NameMapper.cs:7-12):
 * l{i}.ffn_norm when present, l{i}.router and (GLM) l{i}.router_bias as
 * F32 / F16 / BF16 (widened exactly), and as stored (no requantisation) the
 * expert matrices l{i}.e{j}.w_gate / w_up / w_down of the experts the layer
 * holds and l{i}.sw_gate / sw_up / sw_down when it has a shared expert.  A
 * missing tensor is QRM_E_STATE, a wrong shape QRM_E_INVALID, a wrong format
 * QRM_E_FORMAT, a malformed file QRM_E_INVALID. */
int qrm_qw_layer_desc(const char* path, int layer_index, int device, int max_tokens, qrm_layer_desc* out);
int qrm_load_qw(qrm_layer* layer, const char* path, int layer_index);

/* ---- forward ----
 * One MoE layer over T tokens (the reference runs T sequential Forward calls).
 * x [T x d] f32, out [T x d] f32.  Optional outputs (NULL to skip):
 * topk_idx [T x k] int32 (the experts in the reference's sorted order),
 * topk_w [T x k] f32 (their combine weights).  Synchronous.  On a
 * single-GPU layer, batches of at most 256 KiB of rows go through pinned,
 * mapped host staging that the layer allocates on its first such call and
 * keeps until qrm_destroy (at least 256 KiB of inputs and as much of
 * outputs); larger batches and expert-parallel layers copy from the caller's
 * arrays directly. */
int qrm_forward(qrm_layer* layer, const float* x, int T, int flags, float* out,
                int32_t* topk_idx, float* topk_w);
/* Same on device buffers, asynchronous on `stream` (a cudaStream_t; NULL =
 * the layer's own stream).  Call qrm_sync (or synchronise the stream) before
 * reading results; qrm_sync reports device-side errors of earlier forwards. */
int qrm_forward_device(qrm_layer* layer, const float* x_dev, int T, int flags, float* out_dev,
                       int32_t* topk_idx_dev, float* topk_w_dev, void* stream);
int qrm_sync(qrm_layer* layer);
/* Dispatch of the last forward: perm [T*k] lists the assignments
 * a = t*k + j sorted by expert (stable: a ascending inside an expert) and
 * offsets [E+1] delimits each expert's run. */
int qrm_last_dispatch(qrm_layer* layer, int32_t* perm, int32_t* offsets);
/* Router logits [T x E] and normalised input xn [T x d] of the last forward
 * (debug/parity; NULL to skip either). */
int qrm_last_router(qrm_layer* layer, float* logits, float* xn);

/* Per-stage device timing of forwards (CUDA events on the forward's stream).
 * qrm_last_profile fills ms[QRM_STAGE_COUNT] for the last forward
 * (route, topk, dispatch, gate/up, down, combine; stages that did not run
 * report 0) and bytes[QRM_STAGE_COUNT] with the algorithmic HBM bytes of
 * the gate/up and down stages (compressed expert bytes of the experts the
 * batch selected, plus activations).  No counterpart in the reference
 * (its `bench` command times whole tokens, Commands.cs:801-829). */
enum { QRM_STAGE_ROUTE = 0, QRM_STAGE_TOPK, QRM_STAGE_DISPATCH, QRM_STAGE_GATEUP, QRM_STAGE_DOWN,
       QRM_STAGE_COMBINE, QRM_STAGE_COUNT };
int qrm_set_profiling(qrm_layer* layer, int on);
int qrm_last_profile(qrm_layer* layer, float* ms, double* bytes);

/* Number of this library's kernel launches in the last forward (one CUDA
 * graph replay).  No counterpart in the reference. */
int qrm_last_launch_count(qrm_layer* layer, int* count);

/* ---- layer stack: n MoE layers of one shape on a device-resident residual
 * stream (the MoE part of ForwardLegacy, StreamingEngine.cs:213-286: each
 * layer x += MoeFfn(RmsNorm(x)), or what `flags` asks per layer) ----
 * hbm_budget: bytes of expert weights the stack may keep in HBM (0 = no
 * limit).  While every layer fits, all are resident.  Otherwise the first
 * n_resident layers stay resident and the others are kept in pinned host
 * memory and streamed into two device slots by layer parity, each copy
 * overlapping the compute of the layer before (PrefetchPipeline's ping-pong
 * staging, src/QuantRunner.Core/Runtime/PrefetchPipeline.cs:64-166; its
 * over-budget fallback :131-135 becomes streaming from host memory).
 * Uploads go through each layer (qrm_stack_layer + qrm_upload_*, or
 * qrm_stack_load_qw for .qw file layers first_layer ... first_layer+n-1); a
 * streamed layer's expert upload also fills its host image.  The stack owns
 * its layers (do not qrm_destroy them).  qrm_stack_forward_device runs all
 * layers on `stream` (NULL = layer 0's stream): x_dev [T x d] in, out_dev
 * [T x d] out (may alias x_dev); asynchronous; qrm_stack_sync reports
 * device-side errors. */
typedef struct qrm_stack qrm_stack;
int  qrm_stack_create(const qrm_layer_desc* desc, int n_layers, size_t hbm_budget, qrm_stack** out);
void qrm_stack_destroy(qrm_stack* stack);
int  qrm_stack_layer(qrm_stack* stack, int i, qrm_layer** layer);
int  qrm_stack_info(qrm_stack* stack, int* n_resident, size_t* layer_bytes);
int  qrm_stack_load_qw(qrm_stack* stack, const char* path, int first_layer);
int  qrm_stack_forward_device(qrm_stack* stack, const float* x_dev, int T, int flags, float* out_dev, void* stream);
int  qrm_stack_sync(qrm_stack* stack);

/* ---- operator API: DotKernels.MatVecParallel / DotKernels.GEMM on the GPU ----
 * (DotKernels.cs:610-660).  A qrm_matrix holds one [rows x cols] matrix in
 * HBM; qrm_matrix_gemv computes y[t] = W x[t] for T tokens
 * (x_dev [T x cols], y_dev [T x rows]). */
typedef struct qrm_matrix qrm_matrix;
int  qrm_matrix_create(int device, int fmt, int64_t rows, int64_t cols,
                       const void* bytes, size_t nbytes, qrm_matrix** out);
void qrm_matrix_destroy(qrm_matrix* m);
int  qrm_matrix_gemv(qrm_matrix* m, const float* x_dev, int T, float* y_dev, void* stream);

/* ---- dense FFN: StreamingEngine.DenseFfn / DenseFfnOut
 * (src/QuantRunner.Core/Runtime/StreamingEngine.cs:599-622), the FFN of the
 * dense layers of a MoE model (first_k_dense_replace, :633-637), from three
 * matrix operators ----
 * gate, up: [f x d]; down: [d x f], all on one device (the qrm_ffn refers to
 * them; destroy it before them).  qrm_ffn_forward computes, for T <=
 * max_tokens tokens, out = x + W_down SwiGLU(W_gate xn, W_up xn) (DenseFfn,
 * x_dev given) or out = W_down SwiGLU(...) (DenseFfnOut, x_dev NULL), with
 * Glm5Ops.LimitedSwiglu's clamp when swiglu_limit > 0; asynchronous on
 * `stream`.  out_dev may alias x_dev (the engine adds into x in place). */
typedef struct qrm_ffn qrm_ffn;
int  qrm_ffn_create(qrm_matrix* gate, qrm_matrix* up, qrm_matrix* down, int max_tokens, qrm_ffn** out);
void qrm_ffn_destroy(qrm_ffn* ffn);
int  qrm_ffn_forward(qrm_ffn* ffn, const float* xn_dev, const float* x_dev, int T, float swiglu_limit,
                     float* out_dev, void* stream);

/* qrm_matrix_gemv without any device allocation.  No counterpart in the
 * reference.  qrm_matrix_gemv grows the matrix's activation-table buffer when
 * T rises (stream synchronise, cudaFree, cudaMalloc); cudaFree synchronises
 * the whole device, so a caller that overlaps work on several streams, or one
 * that has committed all HBM to weights and caches up front, cannot take that
 * path.  This variant keeps the tables (Q4_K / Q8_0 / Q4_0 matrices) in a
 * fixed 1 MiB device array per device:
 *   - T * (2*cols + 128 + cols/4, rounded up to 16) must be <= 1048576
 *     bytes, else QRM_E_CAPACITY (cols 7168: T <= 64);
 *   - the array is shared by every call on the device: calls that overlap
 *     in time (other streams, other threads, other matrices) race on it;
 *   - the first call on each device looks up the array's address
 *     (cudaGetSymbolAddress) and must come before any stream capture;
 *   - that address is kept for the life of the process: it does not survive
 *     a cudaDeviceReset of the device, after which this entry point must not
 *     be called again in the same process.
 * Nothing needs to start at zero: every table byte read is written first. */
int  qrm_matrix_gemv_static(qrm_matrix* m, const float* x_dev, int T, float* y_dev, void* stream);

/* ---- expert parallelism (no counterpart in the reference, whose MoE layer
 * runs in one process) ----
 * world ranks, one process and GPU each; rank r holds the routed experts
 * [r*E/world, (r+1)*E/world) (qrm_expert_range; uploads of other experts fail
 * with QRM_E_INVALID) and replicas of norm, router and shared expert.  Every
 * rank calls qrm_forward / qrm_forward_device with the same T for its own
 * tokens, the same number of times; the forward routes them (bit-identical on
 * every rank), sends each token to the ranks that hold its experts, runs the
 * local experts for the assignments this rank holds, returns each expert
 * output row to the token's owner, runs the shared expert for the owner's own
 * tokens and combines on the owner in slot order, so the output equals the
 * single-GPU forward bit for bit.  The exchanges are stores into the peers'
 * memory over NVLink (CUDA IPC mappings made at creation: a token row goes
 * only to ranks holding one of its experts, an output row only to its owner)
 * when every rank can map every other rank's memory, else NCCL all-gather and
 * grouped send/recv of fixed-size blocks (QRM_EP_P2P=0 in the environment
 * forces NCCL); a peer
 * that does not deliver within the wait limit (2 s, or QRM_WAIT_LIMIT_US
 * microseconds in the environment when a layer is created) makes qrm_sync return
 * QRM_E_TIMEOUT, after which the layer should be destroyed.  The id comes
 * from qrm_nccl_unique_id on one rank and is passed to every rank by the host
 * (128 bytes); qrm_create_ep returns once all ranks have joined, and
 * qrm_destroy of an expert-parallel layer is collective (it waits up to ~10 s
 * for the other ranks).  qrm_last_profile_ep gives the stage times of an
 * expert-parallel forward (qrm_set_profiling on). */
#define QRM_NCCL_ID_BYTES 128
int qrm_nccl_unique_id(void* id_out);
int qrm_create_ep(const qrm_layer_desc* desc, int rank, int world, const void* nccl_id, qrm_layer** out);
int qrm_expert_range(qrm_layer* layer, int* first, int* count);
/* How the layer exchanges tokens and outputs: 0 single GPU, 1 NCCL, 2 peer
 * memory (NVLink stores). */
#define QRM_EP_SINGLE 0
#define QRM_EP_NCCL 1
#define QRM_EP_PEER 2
int qrm_ep_transport(qrm_layer* layer, int* transport);
/* Per-stage device time (ms) of the last expert-parallel forward, run with
 * qrm_set_profiling(layer, 1): route (RMSNorm, router, own top-k), records
 * (token rows and top-k rows to the experts' ranks, then the dispatch, which
 * waits for every rank's records), gate/up, down, outputs (expert output rows
 * to the tokens' owners), combine (waits for every holder's rows).  A wait on
 * a slower rank counts in the stage that waits. */
enum { QRM_EP_STAGE_ROUTE = 0, QRM_EP_STAGE_RECORDS, QRM_EP_STAGE_GATEUP, QRM_EP_STAGE_DOWN, QRM_EP_STAGE_OUTPUTS,
       QRM_EP_STAGE_COMBINE, QRM_EP_STAGE_COUNT };
int qrm_last_profile_ep(qrm_layer* layer, float* ms);

/* ---- self-tests (no counterpart in the reference; its `selftest` command
 * checks the CPU kernels, src/QuantRunner.Cli/Commands.cs:2257-2325) ----
 * qrm_selftest_expf writes the bits of the routing kernels' binary32 exp of
 * the floats with bit patterns first .. first+count-1 (wrapping) to out_dev
 * [count] (asynchronous on `stream`), for comparison with the C runtime's
 * expf that the reference's MathF.Exp calls.
 * qrm_selftest_waits runs the library's bounded waits on an mbarrier nothing
 * arrives at and on a peer flag nothing raises, with a limit of limit_us
 * (1 us .. 10 s) on `device`; it returns QRM_E_TIMEOUT when they gave up (the
 * expected outcome; gave_up[2] says which did), and the device stays usable. */
int qrm_selftest_expf(uint32_t first, uint32_t count, uint32_t* out_dev, void* stream);
int qrm_selftest_waits(int device, int64_t limit_us, int* gave_up);

/* ---- synthetic weights on the device (the reference's `synthesize`,
 * src/QuantRunner.Cli/Program.cs:247-369) ----
 * qrm_synth_gaussian fills dst_dev[n] with sigma * N(0,1) from a
 * counter-based generator (splitmix64 + Box-Muller); qrm_synth_quantize runs
 * the reference quantiser (BlockQuantizer.cs; fmt 108 = QuantizeTriLegacy)
 * on the device, byte-identical to the CPU one. */
int qrm_synth_gaussian(float* dst_dev, int64_t n, uint64_t seed, float sigma, void* stream);
int qrm_synth_quantize(int fmt, const float* src_dev, int64_t n, void* dst_dev, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* QRMOE_H */
