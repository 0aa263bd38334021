/*
 * ethos_b200.h -- C ABI of the B200-native ETHOS expert layer.
 *
 * The reference (wrmedford/ETHOS) is pure Python: its expert layer is the
 * nn.Module pair SimplifiedHypernetMoE (model.py:267-343) /
 * FusedLowRankMoE_Reordered (kernels.py:123-221) with ProductKeyRouter
 * (model.py:182-254), and its only kernel is the Triton moe_reorder_kernel
 * (kernels.py:18-120) launched from kernels.py:179-215.  The entry points below
 * replace those calls; each cites the reference code it stands in for.  The
 * Python host (ethos_b200/_lib.py) binds them with ctypes.
 *
 * Conventions
 *  - All tensor arguments are raw DEVICE pointers to contiguous row-major
 *    buffers owned by the caller (the library never allocates or frees device
 *    memory); sizes are int64; `stream` is a cudaStream_t (NULL = legacy).
 *  - bf16 buffers hold IEEE bfloat16 values (2 bytes each).
 *  - Every entry point returns an ethos status (0 = OK) and never throws.
 *    Device-side faults of the data (an expert id out of range) and bounded
 *    wait timeouts are recorded in the caller-provided device error word
 *    `dev_err` (an int32, zero-initialised by the caller) and read back with
 *    ethos_read_device_error().
 *  - Calls are stateless and re-entrant; the only process-wide state is a
 *    lazily initialised per-device attribute cache, the launch counter
 *    (ethos_launch_count) and the bounded-wait limit (ethos_set_wait_limit_ns).
 *  - Entry points only launch work on `stream`; they do not synchronise.
 */
#ifndef ETHOS_B200_H
#define ETHOS_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------- status -- */
#define ETHOS_OK 0
#define ETHOS_ERR_INVALID_ARG 1       /* null pointer, negative size          */
#define ETHOS_ERR_UNSUPPORTED_SHAPE 2 /* dims outside the compiled kernels    */
#define ETHOS_ERR_ALIGNMENT 3         /* pointer not 16-byte aligned          */
#define ETHOS_ERR_WORKSPACE 4         /* workspace smaller than required      */
#define ETHOS_ERR_CUDA 5              /* a CUDA runtime call failed           */
#define ETHOS_ERR_TENSOR_MAP 6        /* cuTensorMapEncodeTiled failed        */
#define ETHOS_ERR_NO_DEVICE 7         /* no sm_100 device current             */
#define ETHOS_ERR_SCRATCH_LIMIT 8     /* request exceeds the static scratch   */
/* device-side codes (reported through dev_err) */
#define ETHOS_ERR_ID_OUT_OF_RANGE 16  /* an expert id outside [0, N)          */
#define ETHOS_ERR_TIMEOUT_BASE 1000   /* + site: a bounded wait gave up       */

/* Layer dimensions (names follow the reference config, train.py:33-48). */
typedef struct ethos_dims {
  int64_t tokens;       /* T = batch * seq                                    */
  int64_t d_model;      /* d                                                   */
  int64_t num_experts;  /* N = K * K                                           */
  int64_t num_sub_keys; /* K                                                   */
  int64_t d_query;      /* dq (split into two halves of dq/2)                  */
  int64_t d_latent;     /* dl                                                  */
  int64_t d_hidden;     /* dh = d_intermediate_hypernet                        */
  int64_t num_heads;    /* H = num_routing_heads                               */
  int64_t top_k;        /* k                                                   */
} ethos_dims;

int ethos_abi_version(void);
const char* ethos_status_string(int status);

/* Number of kernels this library has launched in this process, over all
 * devices and streams (a monotonically increasing count, read by benchmarks
 * to report how many of the library's kernels ran in a timed region).  No
 * counterpart in the reference. */
uint64_t ethos_launch_count(void);

/* Copies the device error word to *host_code (synchronising `stream`) and,
 * when reset != 0, clears it. */
int ethos_read_device_error(int* dev_err, int* host_code, int reset, void* stream);

/* Checks `dims` against the compiled kernels; returns ETHOS_OK or
 * ETHOS_ERR_UNSUPPORTED_SHAPE.  Supported: d_latent 128, d_hidden 512,
 * num_heads * top_k <= 128 (multiple of 4), top_k in {4, 8, 16},
 * num_sub_keys a multiple of 32 up to 512 with num_sub_keys >= top_k,
 * d_query/2 a multiple of 32, d_model a multiple of 256,
 * (num_heads * d_query + d_hidden) a multiple of 256. */
int ethos_check_dims(const ethos_dims* dims);

/* --------------------------------------------------------- forward -- */
/* Expert execution paths (argument `expert_path`):
 *  1 = fused per token: gather the selected latent rows, expand them on
 *      tcgen05 and apply GELU in the epilogue (no scratch);
 *  2 = expert table: expand + GELU once per expert into an fp16 [N, dh]
 *      table (scratch), then gather hidden rows per token;
 *  3 = cached expert table: path 2 without the expansion, gathering from a
 *      table the caller built with ethos_expert_table_build (serving with
 *      frozen parameters; the caller rebuilds it whenever expert_latents or
 *      net.0.weight change).  Needs num_heads * top_k >= 16;
 *  0 = automatic: the table once tokens*heads*top_k >= num_experts. */
#define ETHOS_EXPERT_AUTO 0
#define ETHOS_EXPERT_FUSED 1
#define ETHOS_EXPERT_TABLE 2
#define ETHOS_EXPERT_TABLE_CACHED 3

/* Stage boundaries of ethos_layer_forward (indices into stage_events). */
#define ETHOS_STAGE_START 0
#define ETHOS_STAGE_PROJECTION 1   /* after the query + x_proj GEMM            */
#define ETHOS_STAGE_BATCHNORM 2    /* after the training-mode BatchNorm kernels */
#define ETHOS_STAGE_TOPK 3         /* after scoring + top-k + softmax           */
#define ETHOS_STAGE_EXPERT_TABLE 4 /* after the expert-table GEMM (table path)  */
#define ETHOS_STAGE_EXPERTS 5      /* after the per-token expert kernel         */
#define ETHOS_STAGE_END 6          /* after the W_v up-projection GEMM          */
#define ETHOS_STAGE_COUNT 7

/* Scratch bytes needed by ethos_layer_forward / ethos_router_forward. */
size_t ethos_forward_workspace_size(const ethos_dims* dims, int bn_training, int expert_path);

/* Scratch bytes needed by ethos_expert_forward. */
size_t ethos_expert_workspace_size(const ethos_dims* dims, int expert_path);

/* Router + reordered expert forward of one layer.
 *
 * Replaces SimplifiedHypernetMoE.forward (model.py:288-343) and
 * FusedLowRankMoE_Reordered.forward (kernels.py:145-221, including the
 * per-head Triton launches kernels.py:167-217) together with the router call
 * ProductKeyRouter.forward (model.py:208-254).
 *
 *  x         bf16 [T, d]
 *  w_cat     bf16 [H*dq + dh, d]: row block h = query_projs[h].weight
 *            (model.py:195-197); last dh rows = net.2.weight[:d]^T (W_u of
 *            model.py:299, transposed to [dh, d])
 *  bn        fp32 [5, H*dq]: rows = query_projs bias, query_norms weight,
 *            query_norms bias, running_mean, running_var (model.py:195-202).
 *            In training mode the running rows are updated in place
 *            (momentum `bn_momentum`, unbiased variance), as BatchNorm1d does.
 *  key_cat   bf16 [2, K, dq]: [p][key] = sub_keys_{p+1}.weight[key] written
 *            twice ([hi | lo] operand layout of the split-bf16 fp32 scoring)
 *  latents   bf16 [N, dl]   expert_latents.weight
 *  w1        bf16 [dh, dl]  generation_network.net.0.weight
 *  wv        bf16 [d, dh]   generation_network.net.2.weight[d:]
 *  expert_path  ETHOS_EXPERT_AUTO / _FUSED / _TABLE (see above)
 *  y         bf16 [T, d]    output (already divided by H, model.py:341)
 *  ids       int32 [T, H, k] selected expert ids (i1*K + i2, model.py:245)
 *  weights   fp32 [T, H, k]  softmax routing weights (model.py:234, fp32)
 *  stage_events  optional (may be NULL) array of ETHOS_STAGE_COUNT cudaEvent_t:
 *            event i is recorded on `stream` at stage boundary i (below), so a
 *            caller can time each kernel of the real call with no extra sync
 *  save_*    optional (may be NULL) tensors kept for the backward pass:
 *            save_xp fp32 [T, dh] (x @ W_u), save_hacc bf16 [T, dh]
 *            (sum_{h,k} a*h), save_dot fp32 [T, H*k] (h . x_proj),
 *            save_qpre fp32 [T, H*dq] (pre-BatchNorm queries, x Wq^T + b),
 *            save_bn fp32 [2, H*dq] (batch mean, 1/sqrt(var+eps); training only),
 *            save_qs bf16 [2, H, T, dq] (normalised queries per half and head,
 *            split hi | lo),
 *            save_htab, save_gtab fp16 [N, dh] (both or neither; used only
 *            when the table path runs): the expert table H = gelu(E W1^T) is
 *            built there instead of in the workspace, together with
 *            G = gelu'(E W1^T), so that the backward need not rebuild them.
 *            With expert_path ETHOS_EXPERT_TABLE_CACHED, save_htab is instead
 *            the caller's prebuilt table (read only) and save_gtab is NULL.
 */
int ethos_layer_forward(const ethos_dims* dims, const void* x, const void* w_cat, float* bn, float bn_eps,
                        float bn_momentum, int bn_training, const void* key_cat, const void* latents,
                        const void* w1, const void* wv, int expert_path, void* y, int32_t* ids,
                        float* weights, float* save_xp, void* save_hacc, float* save_dot,
                        float* save_qpre, float* save_bn, void* save_qs, void* save_htab, void* save_gtab,
                        void* workspace, size_t workspace_bytes, int* dev_err, void* const* stage_events,
                        void* stream);

/* Router alone: ProductKeyRouter.forward (model.py:208-254) on x [T, d]
 * (bf16).  Arguments as for ethos_layer_forward; w_cat needs only its first
 * H*dq rows.  Outputs ids int32 [T, H, k] and fp32 softmax weights. */
int ethos_router_forward(const ethos_dims* dims, const void* x, const void* w_cat, float* bn, float bn_eps,
                         float bn_momentum, int bn_training, const void* key_cat, int32_t* ids,
                         float* weights, float* save_qpre, float* save_bn, void* workspace,
                         size_t workspace_bytes, int* dev_err, void* stream);

/* Reordered experts alone, given routing decisions (the per-head Triton
 * launches of kernels.py:167-217 / the expert loop of model.py:306-336):
 *  latents bf16 [N, dl]; w1 bf16 [dh, dl]; ids int32 [T, H*k];
 *  weights fp32 [T, H*k]; xp fp32 [T, dh] (x @ W_u)
 *  hacc   bf16 [T, dh] out: sum_{h,k} gelu(h.xp)*w*h;  dot fp32 [T, H*k] out
 *         (optional, may be NULL)
 *  workspace: ethos_expert_workspace_size() bytes (the fp16 expert table for
 *         the table path; may be NULL for the fused path; for
 *         ETHOS_EXPERT_TABLE_CACHED it holds the prebuilt table)
 * Ids outside [0, N) are not dereferenced: they set ETHOS_ERR_ID_OUT_OF_RANGE
 * in dev_err and read row 0 instead. */
int ethos_expert_forward(const ethos_dims* dims, int expert_path, const void* latents, const void* w1,
                         const int32_t* ids, const float* weights, const float* xp, void* hacc, float* dot,
                         void* workspace, size_t workspace_bytes, int* dev_err, void* stream);

/* The expert table alone (no counterpart in the reference, whose experts
 * expand every selection, model.py:320-323): htab fp16 [N, dh] =
 * gelu_erf(latents @ w1^T), and when gtab (fp16 [N, dh], may be NULL) is
 * given also gelu_erf'(latents @ w1^T).  latents bf16 [N, dl], w1 bf16
 * [dh, dl].  The table that ETHOS_EXPERT_TABLE_CACHED gathers from. */
int ethos_expert_table_build(const ethos_dims* dims, const void* latents, const void* w1, void* htab, void* gtab,
                             int* dev_err, void* stream);

/* Router forward that allocates nothing (no counterpart in the reference).
 *
 * For callers that cannot allocate device memory per call: a host that runs
 * under a fixed memory plan reserved at start-up (a serving process that must
 * not grow or fragment its device heap mid-request), or an embedding runtime
 * that hands this library its input and output buffers but owns no device
 * allocator of its own.  Same computation as ethos_router_forward with
 * BatchNorm in eval mode (running statistics); its scratch -- the split-bf16
 * scoring operand and the folded per-column BatchNorm affine -- lives in a
 * file-scope static device array of ETHOS_NOALLOC_SCRATCH_BYTES that every
 * GPU loading this library holds until process exit.
 *  - Limit: tokens * num_heads * d_query * 4 + num_heads * d_query * 8 plus
 *    alignment must fit the array (258 tokens at 8 heads x d_query 512);
 *    larger requests return ETHOS_ERR_SCRATCH_LIMIT and launch nothing.
 *  - The first call on each device looks up the array's device address
 *    (cudaGetSymbolAddress) with that device current; make that first call
 *    before any stream capture.
 *  - All calls share the one array: calls that overlap on the GPU (other
 *    streams, other host threads) race and must be serialised by the caller.
 *    Nothing in the array needs to start zeroed: every call fully rewrites
 *    the parts it reads.
 * Arguments as for ethos_router_forward (x bf16 [T, d], w_cat first H*dq
 * rows, bn fp32 [5, H*dq] read only, key_cat bf16 [2, K, dq]); outputs
 * ids int32 [T, H, k] and fp32 softmax weights [T, H, k]. */
#define ETHOS_NOALLOC_SCRATCH_BYTES (4u * 1024u * 1024u + 64u * 1024u)
int ethos_router_forward_noalloc(const ethos_dims* dims, const void* x, const void* w_cat, const float* bn,
                                 float bn_eps, const void* key_cat, int32_t* ids, float* weights, int* dev_err,
                                 void* stream);

/* Product-key top-k from already normalised queries (the scoring, per-half
 * top-k, candidate-grid top-k, softmax and id decode of model.py:217-245).
 *  q     bf16 [H, T, dq]  normalised queries
 *  keys  bf16 [2, K, dq/2] sub_keys_1.weight, sub_keys_2.weight
 *  ids   int32 [T, H, k];  weights fp32 [T, H, k]
 * Scores are accumulated in fp32 from the bf16 operands. */
int ethos_product_key_topk(const ethos_dims* dims, const void* q, const void* keys, int32_t* ids,
                           float* weights, int* dev_err, void* stream);

/* ------------------------------------------------------- backward -- */
/* Scratch bytes needed by ethos_layer_backward. */
size_t ethos_backward_workspace_size(const ethos_dims* dims);

/* Backward of ethos_layer_forward: the gradients autograd computes through
 * SimplifiedHypernetMoE.forward (model.py:288-343) including the router
 * (model.py:208-254) and its BatchNorm.
 *  dy         [T, d] bf16 (dy_fp32 = 0) or fp32 (dy_fp32 = 1): dL/dy
 *  x, w_cat, bn, key_cat, latents, w1, wv, ids, weights: as passed to /
 *             returned by the forward call; bn_training as in the forward
 *  save_*     the forward's save buffers (all required; save_bn in training)
 *  htab, gtab the forward's save_htab / save_gtab when it filled them (table
 *             path), else NULL: the backward then builds both itself
 * Outputs (fp32 unless stated, overwritten):
 *  dx        [T, d]         fp32, or bf16 when dx_bf16 != 0 (the dx GEMM
 *                           then stores bf16 directly; for a bf16 layer
 *                           input, no separate conversion pass)
 *  d_latents [N, dl]        expert_latents.weight
 *  d_w1      [dh, dl]       generation_network.net.0.weight
 *  d_w2      [2d, dh]       generation_network.net.2.weight
 *  d_wq      [H*dq, d]      query_projs[h].weight stacked
 *  d_bn      [3, H*dq]      query_projs bias, query_norms weight, bias
 *  d_keys    [2, K, dq/2]   sub_keys_1.weight, sub_keys_2.weight */
int ethos_layer_backward(const ethos_dims* dims, int bn_training, float bn_eps, const void* dy, int dy_fp32,
                         const void* x, const void* w_cat, const float* bn, const void* key_cat, const void* latents,
                         const void* w1, const void* wv, const int32_t* ids, const float* weights,
                         const float* save_xp, const void* save_hacc, const float* save_dot, const float* save_qpre,
                         const float* save_bn, const void* save_qs, const void* htab, const void* gtab,
                         void* dx, int dx_bf16, float* d_latents, float* d_w1, float* d_w2, float* d_wq,
                         float* d_bn, float* d_keys, void* workspace, size_t workspace_bytes, int* dev_err,
                         void* const* stage_events, void* stream);

/* Backward stage events: with a non-NULL `stage_events` (ETHOS_BWD_STAGE_COUNT
 * cudaEvent_t, entries may be NULL) the backward records
 *   ETHOS_BWD_STAGE_EXPERTS  once d_latents and d_w1 are final (their
 *                            all-reduce can start while the router and
 *                            BatchNorm gradients are still being computed),
 *   ETHOS_BWD_STAGE_END      after the last gradient kernel. */
#define ETHOS_BWD_STAGE_EXPERTS 0
#define ETHOS_BWD_STAGE_END 1
#define ETHOS_BWD_STAGE_COUNT 2

/* The two halves of ethos_layer_backward as separate calls, for a host that
 * routes with its own router (and so needs expert-only gradients and the
 * gradient with respect to the routing weights) or that runs only the router
 * from this library.  Composed, they give what ethos_layer_backward gives
 * (which fuses the two dx GEMMs into one over [dq | dxp]).
 *
 * ethos_expert_backward: the backward of ethos_expert_forward -- the
 * gradients autograd takes through the expert loop of model.py:306-336 given
 * hacc's gradient.
 *  latents, w1, ids, weights, xp  as passed to ethos_expert_forward
 *  dot       fp32 [T, H*k]  ethos_expert_forward's `dot` output
 *  dhacc     fp32 [T, dh]   dL/dhacc (for y = hacc W_v^T / H: dy W_v / H)
 *  htab, gtab  fp16 [N, dh] tables from ethos_layer_forward's save_htab /
 *            save_gtab, or both NULL (then built in the workspace)
 * Outputs (fp32, overwritten):
 *  dxp       [T, dh]        dL/dxp (the caller applies W_u: dx = dxp W_u^T)
 *  d_weights [T, H*k]       dL/d(routing weight), the input of the router's
 *                           backward (model.py:234's softmax output)
 *  d_latents [N, dl], d_w1 [dh, dl]
 * Ids outside [0, N) set ETHOS_ERR_ID_OUT_OF_RANGE in dev_err. */
size_t ethos_expert_backward_workspace_size(const ethos_dims* dims);
int ethos_expert_backward(const ethos_dims* dims, const void* latents, const void* w1, const int32_t* ids,
                          const float* weights, const float* xp, const float* dot, const float* dhacc,
                          const void* htab, const void* gtab, float* dxp, float* d_weights, float* d_latents,
                          float* d_w1, void* workspace, size_t workspace_bytes, int* dev_err, void* stream);

/* ethos_router_backward: the backward of ethos_router_forward
 * (ProductKeyRouter.forward, model.py:208-254, under autograd): softmax
 * backward into the selected grid scores, sub-key and query gradients, the
 * BatchNorm backward (batch statistics when bn_training, else running
 * statistics), and the query projection's gradients.
 *  x, w_cat, bn, key_cat, ids, weights  as passed to / returned by the forward
 *            (w_cat needs only its first H*dq rows)
 *  d_weights fp32 [T, H*k]  dL/d(routing weight)
 *  save_qpre, save_bn       the forward's save buffers (save_bn in training);
 *            the normalised queries are recomputed from them
 * Outputs (fp32):
 *  dx        [T, d]         overwritten, or added to when accumulate_dx != 0
 *                           (to sum the router's and the experts' shares)
 *  d_wq [H*dq, d], d_bn [3, H*dq], d_keys [2, K, dq/2]  overwritten */
size_t ethos_router_backward_workspace_size(const ethos_dims* dims);
int ethos_router_backward(const ethos_dims* dims, int bn_training, float bn_eps, const void* x, const void* w_cat,
                          const float* bn, const void* key_cat, const int32_t* ids, const float* weights,
                          const float* d_weights, const float* save_qpre, const float* save_bn, float* dx,
                          int accumulate_dx, float* d_wq, float* d_bn, float* d_keys, void* workspace,
                          size_t workspace_bytes, int* dev_err, void* stream);

/* Plain bf16 GEMM D[M, N] = A[M, K] B[N, K]^T * scale on the tcgen05 path
 * (fp32 accumulate), used by the layer and exposed for tests.  out_dtype 0 =
 * fp32, 1 = bf16.  M >= 1, N % 128 == 0, K % 8 == 0. */
int ethos_gemm_bf16(const void* a, const void* b, void* d, int64_t M, int64_t N, int64_t K, float scale,
                    int out_dtype, int* dev_err, void* stream);

/* General form: D[m, n] (=|+=) scale * sum_k A(m, k) B(n, k).
 *  a_mn_major = 0: A stored [M][K] (row pitch lda); 1: A stored [K][M]
 *  b_mn_major = 0: B stored [N][K] (row pitch ldb); 1: B stored [K][N]
 *  out_mode 0: D fp32 = ..., 1: D bf16 = ..., 2: D fp32 += ... (atomic,
 *  split-K over K when the output has few tiles); D row pitch ldd.
 * Row pitches and base pointers must be 16-byte aligned. */
int ethos_gemm_bf16_ex(const void* a, int64_t lda, int a_mn_major, const void* b, int64_t ldb, int b_mn_major,
                       void* d, int64_t ldd, int64_t M, int64_t N, int64_t K, float scale, int out_mode,
                       int* dev_err, void* stream);

/* ------------------------------------------------------ fp32 arithmetic --
 * The same layer computed in fp32, for modules whose parameters are fp32 (the
 * reference's SimplifiedHypernetMoE / ProductKeyRouter, model.py:208-343,
 * then run entirely in fp32).  Contractions use the tcgen05 GEMMs on
 * split-bf16 operands (v = hi + lo, products hi*hi + lo*hi + hi*lo with fp32
 * accumulation: about 2^-16 relative error per product); BatchNorm, scores,
 * top-k, softmax, the expert table (fp32, rebuilt every call), GELU and all
 * reductions stay fp32.  Extra shape rule: d_query / 2 a multiple of 128.
 * Same argument meanings as the bf16 entry points, with fp32 tensors:
 *  x [T, d]; w_cat [H*dq + dh, d] (only the first H*dq rows when y is NULL);
 *  keys [2, K, dq/2] = sub_keys_1.weight, sub_keys_2.weight (NOT doubled);
 *  latents [N, dl]; w1 [dh, dl]; wv [d, dh]; y [T, d] or NULL for the router
 *  alone (ProductKeyRouter.forward, model.py:208-254: then latents, w1, wv
 *  and every save_* may be NULL).  save_qhat [2, H, T, dq/2] holds the
 *  normalised query halves; save_htab / save_gtab [N, dh] the expert table
 *  and its GELU derivative (save_gtab needs save_htab). */
size_t ethos_forward_workspace_size_f32(const ethos_dims* dims, int bn_training);
int ethos_layer_forward_f32(const ethos_dims* dims, const float* x, const float* w_cat, float* bn, float bn_eps,
                            float bn_momentum, int bn_training, const float* keys, const float* latents,
                            const float* w1, const float* wv, float* y, int32_t* ids, float* weights,
                            float* save_xp, float* save_hacc, float* save_dot, float* save_qpre, float* save_bn,
                            float* save_qhat, float* save_htab, float* save_gtab, void* workspace,
                            size_t workspace_bytes, int* dev_err, void* stream);

/* Backward of ethos_layer_forward_f32 (autograd through model.py:208-343 in
 * fp32): dy fp32 [T, d], the forward's inputs and save buffers (save_bn in
 * training; htab / gtab may be NULL together, the backward then rebuilds
 * them); outputs and stage events as for ethos_layer_backward. */
size_t ethos_backward_workspace_size_f32(const ethos_dims* dims);
int ethos_layer_backward_f32(const ethos_dims* dims, int bn_training, float bn_eps, const float* dy, const float* x,
                             const float* w_cat, const float* bn, const float* keys, const float* latents,
                             const float* w1, const float* wv, const int32_t* ids, const float* weights,
                             const float* save_xp, const float* save_hacc, const float* save_dot,
                             const float* save_qpre, const float* save_bn, const float* save_qhat, const float* htab,
                             const float* gtab, float* dx, float* d_latents, float* d_w1, float* d_w2, float* d_wq,
                             float* d_bn, float* d_keys, void* workspace, size_t workspace_bytes, int* dev_err,
                             void* const* stage_events, void* stream);

/* ------------------------------------------------- failure detection --
 * Every wait inside the kernels (an mbarrier phase: a TMA copy landing, an
 * MMA completing, an accumulator released) is bounded.  A wait that runs out
 * records ETHOS_ERR_TIMEOUT_BASE + site in dev_err; the CTA then drains its
 * in-flight copies and MMAs, frees its tensor memory and exits, leaving the
 * CUDA context usable.  No counterpart in the reference, whose kernels have no
 * waits. */

/* Sets the wait limit of the CURRENT device in nanoseconds (0 restores the
 * default of 2 s).  Synchronises the device.  Affects every later launch on
 * that device, so change it only while no other work of this library runs. */
int ethos_set_wait_limit_ns(uint64_t limit_ns);

/* Test of the bounded waits: the plain GEMM D fp32 [M, N] = A bf16 [M, K] @
 * B bf16 [N, K]^T on the one-SM kernel, with the operand loads of work unit
 * `hold_unit` (a 128 x 128 output tile; unit 0 is the top-left tile) never
 * issued.  The MMA issuer and the epilogue warps of that CTA wait for them
 * until the wait limit runs out, then record ETHOS_ERR_TIMEOUT_BASE + site in
 * dev_err and exit; the other tiles complete.  M >= 1, N % 128 == 0,
 * K % 8 == 0. */
int ethos_test_gemm_withhold(const void* a, const void* b, float* d, int64_t M, int64_t N, int64_t K,
                             int64_t hold_unit, int* dev_err, void* stream);

/* Test of the device GELU (no counterpart in the reference, which calls
 * torch's erf GELU, model.py:323,329): evaluates, on x fp32 [n] (n even, both
 * buffers 16-byte aligned), the erf-form GELU and its derivative exactly as
 * the kernels do, into out fp32 [5, n]: row 0 the scalar form (fused expert
 * path), row 1 the packed-pair form (expert-table epilogue), rows 2 and 3 the
 * value and derivative of the backward tables' form, row 4 the scalar
 * derivative. */
int ethos_test_gelu(const float* x, float* out, int64_t n, void* stream);

/* ------------------------------------------------------ optimizer step --
 * Fused AdamW over many tensors in one launch, the update the reference's
 * training runs through DeepSpeed (train.py:68-104: AdamW, ZeRO-2 with bf16
 * weights and fp32 master copies).  Per element, exactly
 * torch.optim.AdamW(weight_decay=wd) at step `step` (>= 1):
 *   p <- p (1 - lr wd);  m <- m + (1 - b1)(g - m);  v <- b2 v + (1 - b2) g^2
 *   p <- p - (lr / (1 - b1^step)) m / (sqrt(v) / sqrt(1 - b2^step) + eps)
 * `p` is `master` (fp32) when given, whose new value is then also written to
 * `param` rounded to its dtype; otherwise `param` itself (fp32 or bf16).
 * `tensors` is a DEVICE array of `num_tensors` descriptors; `max_n` is the
 * largest `n` among them (sizes the launch).  Grad dtype: fp32 or bf16.
 * `grad_scale` (device fp32 [1], or NULL for 1): every gradient is multiplied
 * by grad_scale[0] before the update (the clip coefficient below). */
typedef struct ethos_adam_tensor {
  void* param;        /* fp32 or bf16 [n]                                     */
  const void* grad;   /* fp32 or bf16 [n]                                     */
  float* exp_avg;     /* fp32 [n]                                             */
  float* exp_avg_sq;  /* fp32 [n]                                             */
  float* master;      /* fp32 [n] or NULL                                     */
  int64_t n;
  int32_t param_bf16; /* 1 if param is bf16                                   */
  int32_t grad_bf16;  /* 1 if grad is bf16                                    */
} ethos_adam_tensor;

int ethos_adamw_step(const ethos_adam_tensor* tensors, int num_tensors, int64_t max_n, float lr, float beta1,
                     float beta2, float eps, float weight_decay, int64_t step, const float* grad_scale, int* dev_err,
                     void* stream);

/* Global-norm gradient clipping, the reference's `gradient_clipping: 1.0`
 * (train.py:100, applied by DeepSpeed before its AdamW step) with the rule of
 * torch.nn.utils.clip_grad_norm_: over every `grad` of `tensors` (the same
 * DEVICE descriptor array as ethos_adamw_step),
 *   norm = sqrt(sum of g^2),  coef = min(1, max_norm / (norm + 1e-6)),
 * written to out fp32 [2] (device) = {norm, coef}; pass &out[1] as
 * ethos_adamw_step's `grad_scale` to clip inside the update (the gradients
 * themselves are not modified).  The sum is taken in a fixed order (fp64
 * partials per block of a fixed grid in `workspace`), so equal gradients give
 * bit-identical results on every GPU.  `workspace`: 8-byte aligned device
 * memory of at least ethos_grad_clip_workspace_size() bytes. */
size_t ethos_grad_clip_workspace_size(void);
int ethos_grad_clip_coef(const ethos_adam_tensor* tensors, int num_tensors, float max_norm, void* workspace,
                         size_t workspace_bytes, float* out, int* dev_err, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ETHOS_B200_H */
