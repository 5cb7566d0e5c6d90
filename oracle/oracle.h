/*
 * oracle.h -- CPU restatement of QuantRunner's MoE FFN hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the CUDA
 * path and the timed CPU baseline ("port" kind).  Nothing in the product
 * (qauntrunner_b200/, include/qrmoe.h) links, loads or calls it; only tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference legs do.
 *
 * Every function restates one C# routine of the reference (paths relative to
 * the QuantRunner project root) and follows its operation order exactly:
 * Vector256 lane semantics are written as explicit 8-lane arrays, C# float
 * expressions are evaluated left to right with every product and sum rounded
 * separately (built with -ffp-contract=off, no -ffast-math), MathF.Round is
 * rintf (ties to even), MathF.Sqrt is sqrtf and MathF.Exp is the C runtime's
 * expf (what .NET 8 calls on Linux).
 *
 * Parity pins: the decoder known-answer blocks of src/QuantRunner.Cli/
 * Commands.cs:2257-2325 and the f16 edge cases of tests/QuantRunner.Tests/
 * Program.cs:60-83 (tests/test_oracle_kat.py).  Not pinned by any reference
 * test: the sort order of exactly tied router scores for more than 16 experts
 * (.NET introsort is unstable there; this oracle uses value descending, index
 * ascending) and the Q4_0 / TRI / routing values (pinned here by hand-computed
 * known answers from the decoder formulas).
 */
#ifndef QRM_ORACLE_H
#define QRM_ORACLE_H
#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* QuantFormat ids, src/QuantRunner.Core/Dtypes.cs:6-26 */
enum { ORC_F32 = 0, ORC_F16 = 1, ORC_BF16 = 2, ORC_Q4_0 = 3, ORC_Q8_0 = 4,
       ORC_Q2_K = 5, ORC_Q4_K = 6, ORC_Q6_K = 7, ORC_TRI = 8, ORC_I8_BLK = 9, ORC_Q3_K = 10,
       ORC_Q5_K = 11, ORC_B1 = 12, ORC_B1X = 13, ORC_T1E = 14, ORC_T1E_LO = 15 };

/* Dtypes.cs:38-65 */
int     orc_block_spec(int fmt, int* block_size, int* block_bytes);
int64_t orc_tensor_bytes(int64_t n, int fmt);

/* Dtypes.cs:76-139 */
float    orc_f16_to_f32(uint16_t h);
uint16_t orc_f32_to_f16(float f);
float    orc_bf16_to_f32(uint16_t b);
uint16_t orc_f32_to_bf16(float f);
void     orc_f32_to_f16_batch(const float* x, uint16_t* y, int64_t n);

/* BlockQuantizer.cs: Q4_0 69-93, Q8_0 97-116, Q4_K 248-318, Q6_K 398-446,
 * TRI 456-521.  fmt 108 selects QuantizeTriLegacy 525-550.  Returns 0 or -1. */
int orc_quantize(int fmt, const float* src, int64_t n, uint8_t* dst);
/* BlockDequantizer.cs: Q4_0 52-69, Q8_0 71-84, Q2_K 87-114, Q3_K 117-151,
 * Q4_K 168-195, Q5_K 198-226, Q6_K 228-256, TRI 258-276, I8_BLK 278-290,
 * B1 299-313, B1X 315-336, T1E / T1E_LO 338-359 (rANS: EntropyCoder.Decode3,
 * EntropyCoder.cs:83-110; -1 where the reference throws); F32/F16/BF16 via
 * Dtypes. */
int orc_dequantize(int fmt, const uint8_t* src, int64_t n, float* dst);

/* DotKernels.DotRow (DotKernels.cs:24-46) with the Vector256 paths of
 * DotF32 51-54 / DotQ4_0 132-179 / DotQ8_0 184-205 / DotQ2_K 240-266 /
 * DotQ3_K 280-318 / DotQ4_K 325-357 / DotQ5_K 378-418 / DotQ6_K 423-451 /
 * DotTri 456-471 / DotI8Blk 476-495 / DotB1 515-531 / DotB1X 533-556 /
 * DotT1E 572-593. */
float orc_dot_row(int fmt, const uint8_t* w, const float* x, int cols);
/* DotKernels.MatVec 599-607 (sequential). */
int orc_matvec(int fmt, const uint8_t* w, int64_t rows, int64_t cols,
               const float* x, float* y);
/* DotKernels.MatVecParallel 610-629: static row chunks over `threads`
 * workers (ProcessorCount-1 in the reference), serial below 16 rows or 1 MiB. */
int orc_matvec_parallel(int fmt, const uint8_t* w, int64_t rows, int64_t cols,
                        const float* x, float* y, int threads);

/* TransformerOps.RmsNorm, TransformerOps.cs:12-40 (w may be NULL). */
void orc_rmsnorm(const float* x, const float* w, float* out, int n, float eps);
/* SimdMath.DotF32, SimdMath.cs:34-53 */
float orc_dot_f32(const float* a, const float* b, int n);
/* MathF.Exp -> C runtime expf, batched. */
void orc_expf_batch(const float* x, float* y, int64_t n);

/* MoeFfn softmax + SelectTopK, StreamingEngine.cs:642-652,801-810.
 * probs (len E, optional) receives the softmax.  k <= 8. */
void orc_route_softmax(const float* logits, int E, int k, int32_t* sel,
                       float* wsel, float* probs);
/* GlmMoeFfn routing, StreamingEngine.cs:730-767 + SelectTopKIndices 793-799.
 * bias may be NULL. */
void orc_route_sigmoid(const float* logits, const float* bias, int E, int k,
                       float routed_scale, int32_t* sel, float* wsel);
/* Canonical dispatch permutation (the reference runs experts per token and
 * has none): stable counting sort of assignments a = t*k + j by expert id.
 * perm[pos] = a, inv_perm[a] = pos, offsets[E+1]. */
void orc_dispatch(const int32_t* sel, int T, int k, int E, int32_t* perm,
                  int32_t* inv_perm, int32_t* offsets);

/* SiluMulInPlace (TransformerOps.cs:114-121) / LimitedSwiglu (Glm5Ops.cs:243-256). */
void orc_swiglu(float* g, const float* u, int n, float limit);

/* Layer description: the ModelConfig MoE fields (ModelConfig.cs:22-61). */
typedef struct orc_moe_desc {
    int32_t d_model, n_experts, n_active, expert_ffn;
    int32_t moe_sigmoid;   /* 1 = GlmMoeFfn, 0 = MoeFfn / LegacyMoeInto */
    float   routed_scale;
    int32_t n_shared;      /* GLM shared expert present when > 0 */
    float   swiglu_limit;
    float   rms_eps;
} orc_moe_desc;

typedef struct orc_moe_weights {
    const float*   norm_w;        /* l{i}.ffn_norm [d] (NULL = no weight)   */
    const float*   router;        /* l{i}.router [E x d] f32                */
    const float*   router_bias;   /* l{i}.router_bias [E] or NULL           */
    const float*   logit_offset;  /* harness-only per-expert offset or NULL */
    const uint8_t* const* gate;   /* [E] l{i}.e{j}.w_gate  [f x d]         */
    const uint8_t* const* up;     /* [E] l{i}.e{j}.w_up    [f x d]         */
    const uint8_t* const* down;   /* [E] l{i}.e{j}.w_down  [d x f]         */
    int32_t fmt_gate, fmt_up, fmt_down;
    const uint8_t* sh_gate;       /* l{i}.sw_gate / sw_up / sw_down or NULL */
    const uint8_t* sh_up;
    const uint8_t* sh_down;
    int32_t fmt_sh_gate, fmt_sh_up, fmt_sh_down;
} orc_moe_weights;

enum { ORC_APPLY_NORM = 1, ORC_ADD_RESIDUAL = 2 };

/* One MoE layer over T tokens, one token at a time as StreamingEngine.Forward
 * does.  flags: ORC_APPLY_NORM computes xn = RmsNorm(x, norm_w) first
 * (StreamingEngine.cs:259-260 / 320-321); ORC_ADD_RESIDUAL selects MoeFfn
 * (626-667: out = x + sum w_j y_j), otherwise LegacyMoeInto (670-712) or,
 * with moe_sigmoid, GlmMoeFfn (720-790).  Optional outputs may be NULL.
 * threads: MatVecParallel worker count (<= 1 runs MatVec serially). */
int orc_moe_forward(const orc_moe_desc* desc, const orc_moe_weights* w,
                    const float* x, int T, int flags, float* out,
                    int32_t* topk_idx, float* topk_w, float* logits_out,
                    float* xn_out, int threads);

/* The routing part of orc_moe_forward alone (RMSNorm, router logits, top-k
 * and combine weights; StreamingEngine.cs:259-260, 639-652, 727-767), for
 * batches whose expert products are checked on a sample of tokens. */
int orc_moe_route(const orc_moe_desc* desc, const orc_moe_weights* w,
                  const float* x, int T, int flags, int32_t* topk_idx,
                  float* topk_w, float* logits_out, float* xn_out, int threads);

#ifdef __cplusplus
}
#endif
#endif
