/*
 * moe_b200.h -- C ABI of libmoe_b200.so, the B200 (sm_100a) MoE FFN layer.
 *
 * This is the drop-in boundary for the MoE hot path of
 * songsnim/accelerating-MoE-inference.  Each entry point names the reference
 * interface it replaces.  Plain pointers and sizes only: device pointers are
 * CUDA device addresses, streams are cudaStream_t passed as void*.
 *
 * Conventions (mirroring the reference's, include/layer.h:29-36):
 *   - x and y are fp32, row-major [T][d_model].
 *   - Expert weights are nn.Linear layout: w1 (gate) and w3 (up) are
 *     [d_ff][d_model], w2 (down) is [d_model][d_ff]; the router weight is
 *     [num_experts][d_model] (src/layer.cu:28-30, 73-77).
 *   - Every function returns MOE_OK (0) or a negative MoeStatus; the message
 *     of the last failure on the calling thread is moe_last_error().  The
 *     reference throws std::invalid_argument / std::runtime_error for the
 *     same conditions (src/tensor.cu:138, src/model_loader.cu:34-42); the C++
 *     layer in include/layer.h rethrows them that way.
 *   - A handle owns its device weights and workspace.  One handle serves one
 *     stream at a time; calls on one handle must not overlap.
 */
#ifndef MOE_B200_H
#define MOE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MOE_B200_ABI_VERSION 1

typedef enum MoeStatus {
    MOE_OK = 0,
    MOE_ERR_INVALID = -1,     /* bad argument or shape */
    MOE_ERR_UNSUPPORTED = -2, /* valid but not supported by this build */
    MOE_ERR_CUDA = -3,        /* a CUDA runtime/driver call failed */
    MOE_ERR_OOM = -4,         /* device or pinned allocation failed */
    MOE_ERR_IO = -5,          /* model.bin missing, truncated or malformed */
    MOE_ERR_TIMEOUT = -6,     /* a bounded device-side wait ran out */
    MOE_ERR_NCCL = -7         /* expert-parallel exchange failed */
} MoeStatus;

/* Routing policy.
 * PHI_QUANTISED: the reference's router, src/layer.cu:47-70 (scores
 *   quantised to router_quantum, top-2 with router_tie_eps hysteresis, lower
 *   index wins, weights 0.5/0.5).  Requires top_k == 2.
 * SOFTMAX_TOPK: softmax over experts, top-k by logit (exact ties go to the
 *   lower expert index), the k weights renormalised to sum to 1. */
typedef enum MoeRouterPolicy {
    MOE_ROUTER_PHI_QUANTISED = 0,
    MOE_ROUTER_SOFTMAX_TOPK = 1
} MoeRouterPolicy;

/* Expert-FFN arithmetic.  The router is always exact fp32 (a k-ascending
 * fused-multiply-add chain, bit-identical to src/tensor.cu:136-148 as the
 * reference's Makefile builds it).
 * FP32: fp32-faithful.  Prefill runs 3xTF32 on tcgen05 tensor cores
 *   (hi*hi + hi*lo + lo*hi into an fp32 TMEM accumulator); decode streams the
 *   fp32 weights through CUDA cores.  Relative L2 error vs the reference
 *   <= 1e-3.
 * BF16: weights and activations rounded to bf16 (RNE), fp32 accumulation.
 *   Relative L2 error vs the reference <= 2e-2.
 * FP32_BF16X3: fp32-faithful at bf16 tensor-core rate.  Every fp32 operand x
 *   is split into bf16 parts hi = bf16(x) and lo = bf16(x - hi) (16
 *   significant bits together), and three bf16 MMAs (hi*hi + hi*lo + lo*hi)
 *   accumulate into the fp32 TMEM accumulator; the dropped lo*lo term and the
 *   split's remainder are about 2^-16 of each product.  Decode streams the
 *   fp32 weights as in FP32.  Relative L2 error vs the reference <= 1e-3.
 *   Not available to the toy decoder (moe_decoder_*). */
typedef enum MoePrecision {
    MOE_PREC_FP32 = 0,
    MOE_PREC_BF16 = 1,
    MOE_PREC_FP32_BF16X3 = 2
} MoePrecision;

/* Tiling of the tcgen05 grouped expert GEMMs.
 * AUTO: CTA_PAIR when the experts average at least 256 routed rows (prefill),
 *   SINGLE_CTA below that (decode-sized T, where most of a 256-row tile would
 *   be padding).
 * SINGLE_CTA: 128 x 256 tiles, one CTA per SM.
 * CTA_PAIR: 256 x 256 tiles on 2-CTA clusters (tcgen05 cta_group::2), each SM
 *   loading half of every weight tile, at every size. */
typedef enum MoeGemmVariant {
    MOE_GEMM_AUTO = 0,
    MOE_GEMM_SINGLE_CTA = 1,
    MOE_GEMM_CTA_PAIR = 2
} MoeGemmVariant;

#define MOE_DECODE_AUTO (-1)

/* Expert-parallel exchange.
 * P2P (default): fused and deduplicated -- each token row is stored once
 *   into the receive buffer of every rank holding any of its experts (over
 *   NVLink, with its selections on that rank as metadata); that rank sums
 *   the weighted outputs of its experts for the row and stores one row back;
 *   completion is signalled with flags in peer memory.  Needs all ranks on
 *   one node (CUDA IPC) and at most 32 ranks.
 * NCCL: separate grouped ncclSend / ncclRecv exchanges after the dispatch
 *   and after the down GEMM, with a host read of the counts in between. */
typedef enum MoeEpTransport {
    MOE_EP_TRANSPORT_P2P = 0,
    MOE_EP_TRANSPORT_NCCL = 1
} MoeEpTransport;

typedef struct MoeConfig {
    int32_t d_model;        /* hidden size; multiple of 64 */
    int32_t d_ff;           /* expert intermediate size (any; padded internally) */
    int32_t num_experts;    /* 1..256 */
    int32_t top_k;          /* 1..min(8, num_experts) */
    int32_t router_policy;  /* MoeRouterPolicy */
    int32_t precision;      /* MoePrecision */
    float router_quantum;   /* PHI policy score quantum (reference 1e-3, include/config.h:22) */
    float router_tie_eps;   /* PHI policy tie margin (reference 2e-2, include/config.h:23) */
    int32_t decode_max_tokens; /* T <= this takes the weight-streaming decode kernels
                                  (0..64; 0: never; MOE_DECODE_AUTO (-1, the
                                  default): the measured crossover for the
                                  precision -- 1 in BF16, 14 in FP32) */
    int32_t device;         /* CUDA device ordinal the handle lives on */
    int32_t max_tokens;     /* workspace is pre-sized for this many tokens; grows on demand */
    int32_t gemm_variant;   /* MoeGemmVariant of the grouped expert GEMMs */
    int32_t ep_transport;   /* MoeEpTransport (expert-parallel handles only) */
    int32_t ep_wait_ms;     /* bound on each peer wait of the fused expert-parallel
                               transport, in ms (0: the default, 5000) */
    int32_t reserved[2];
} MoeConfig;

/* Host fp32 weights of one layer (the tensors PhiMoE loads by name,
 * src/layer.cu:73-77: block_sparse_moe.gate.weight and
 * block_sparse_moe.experts.{e}.w{1,2,3}.weight). */
typedef struct MoeWeightsHost {
    const float* router_weight;      /* [E][d] */
    const float* router_bias;        /* [E] or NULL (added after the dot product) */
    const float* const* w1;          /* E pointers, each [d_ff][d] */
    const float* const* w3;          /* E pointers, each [d_ff][d] */
    const float* const* w2;          /* E pointers, each [d][d_ff] */
} MoeWeightsHost;

typedef struct MoeHandle MoeHandle;

/* Library ABI version (MOE_B200_ABI_VERSION). */
int moe_abi_version(void);

/* Message of the last failure on this thread ("" if none). */
const char* moe_last_error(void);

/* Fill *cfg with defaults: the reference's Phi-tiny-MoE constants
 * (include/config.h:8-23: d 4096, d_ff 448, 16 experts, top-2, PHI policy,
 * quantum 1e-3, tie-eps 2e-2), FP32 precision, device 0. */
void moe_config_init(MoeConfig* cfg);

/* Build a layer from host weights.  Replaces the weight upload of
 * PhiMoE::PhiMoE (src/layer.cu:72-78) and DeviceMoE::DeviceMoE
 * (src/model.cu:1491-1513). */
int moe_create(const MoeConfig* cfg, const MoeWeightsHost* weights, MoeHandle** out);

/* The same, with every pointer in *weights a device address on cfg->device
 * (for callers whose weights are already resident, e.g. generated or loaded
 * on the GPU).  The handle keeps its own converted copies; the caller's
 * buffers may be freed afterwards. */
int moe_create_from_device(const MoeConfig* cfg, const MoeWeightsHost* weights, MoeHandle** out);

/* Build a layer straight from a model.bin (ModelLoader format,
 * src/model_loader.cu:14-50), layer `layer_idx`.  Zero d_model / d_ff /
 * num_experts in *cfg are inferred from the file. */
int moe_create_from_model_bin(const MoeConfig* cfg, const char* path, int layer_idx,
                              MoeHandle** out);

void moe_destroy(MoeHandle* h);

int moe_get_config(const MoeHandle* h, MoeConfig* cfg);

/* Device bytes held by the handle (weights + workspace). */
size_t moe_device_bytes(const MoeHandle* h);

/* Change the decode threshold (MoeConfig.decode_max_tokens) of a handle;
 * MOE_DECODE_AUTO re-selects the precision's default.  moe_get_config
 * reports the threshold in force. */
int moe_set_decode_max_tokens(MoeHandle* h, int32_t max_tokens);

/* y[T][d] = MoE(x[T][d]) on device buffers, enqueued on `stream`; no host
 * synchronisation.  Replaces the device MoE segment src/model.cu:1976-2019
 * (gemm_gate -> route_count/scan/place -> gemm_grouped ->
 * gemm_grouped_combine).  y must not alias x.  T == 0 is a no-op. */
int moe_forward_device(MoeHandle* h, const float* x, float* y, int32_t T, void* stream);

/* The same on host buffers (copies in, computes, copies out, synchronises).
 * Replaces PhiMoE::forward(const Tensor& x, Tensor& y) (src/layer.cu:80-103).
 * Batches of 4096+ tokens run as a pipeline of up to 4 chunks (>= 2048 tokens
 * each) so the host<->device copies overlap the compute; page-locked x and y
 * (moe_host_alloc, Tensor::Alloc::Pinned) are needed for the overlap. */
int moe_forward_host(MoeHandle* h, const float* x, float* y, int32_t T);

/* ---- The MoE half of the decoder layer (PhiDecoderLayer::forward,
 * src/layer.cu:157-161):  y = attn + MoE(layer_norm(attn)).
 *
 * moe_set_post_norm attaches the layer's post_attention_layernorm weight and
 * bias ([d_model] fp32, host pointers, copied) and eps (the reference uses
 * NORM_EPS = 1e-5, include/config.h:19); it replaces the post_norm_weight_ /
 * post_norm_bias_ members of PhiDecoderLayer (src/layer.cu:140-147).
 * moe_create_from_model_bin attaches them by itself when the file holds
 * model.layers.<i>.post_attention_layernorm.{weight,bias} (eps 1e-5).
 *
 * moe_block_forward_device / _host then run the norm's statistics with the
 * reference's serial arithmetic (tensor_ops::layer_norm, src/tensor.cu:
 * 174-189, bit for bit), apply the norm inside the router and the dispatch
 * permute (the normalised activations are never stored), run the MoE, and
 * add the residual after the combine: y = (sum of weighted expert outputs)
 * + attn, in the reference's order.  MOE_ERR_INVALID if no norm is attached.
 * y must not alias attn.  d_model must be a multiple of 128. */
int moe_set_post_norm(MoeHandle* h, const float* weight, const float* bias, float eps);
/* The same block with an RMSNorm in place of the LayerNorm (BASELINE
 * config 4's decoder, which has no counterpart in the reference's Phi
 * model): y = attn + MoE(rms_norm(attn)), rms_norm(x)_j = (x_j * inv) * w_j
 * with inv = 1 / sqrt(sum_j x_j^2 / d_model + eps), the sum of squares in
 * fp32.  weight is [d_model] fp32 (host or device pointer, copied).  Replaces an
 * attached LayerNorm, and moe_set_post_norm replaces this. */
int moe_set_post_rms_norm(MoeHandle* h, const float* weight, float eps);
int moe_block_forward_device(MoeHandle* h, const float* attn, float* y, int32_t T, void* stream);
int moe_block_forward_host(MoeHandle* h, const float* attn, float* y, int32_t T);

/* tensor_ops::layer_norm (src/tensor.cu:174-189) on device buffers, bit for
 * bit with the reference's host function: y[rows][cols] = layer_norm(x) with
 * weight/bias [cols].  Needs no handle; runs on the current device, on
 * `stream`.  cols a multiple of 128; all pointers 16-byte aligned; y may
 * alias x. */
int moe_layer_norm_device(const float* x, const float* weight, const float* bias, float eps,
                          int32_t rows, int32_t cols, float* y, void* stream);

/* Router only, device buffers: logits [T][E] (may be NULL), expert indices
 * and weights [T][top_k] in selection order.  Replaces the router GEMM and
 * route (src/layer.cu:84-91; src/model.cu:505-616, 878-942). */
int moe_route_device(MoeHandle* h, const float* x, int32_t T, float* logits, int32_t* idx,
                     float* weights, void* stream);

/* Router only, host buffers (copies x in, synchronises): logits [T][E] (may
 * be NULL), expert indices and weights [T][top_k].  The host-side view of
 * PhiMoE::route (src/layer.cu:47-70) over a whole batch. */
int moe_route_host(MoeHandle* h, const float* x, int32_t T, float* logits, int32_t* idx,
                   float* weights);

/* Failure-detection self-test.  Every device-side wait in the kernels
 * (mbarrier waits of the TMA / MMA / epilogue pipelines) is bounded in
 * wall-clock time; when one runs out the kernel records an error flag, stops
 * issuing work, drains what it issued and returns, and the host reports
 * MOE_ERR_TIMEOUT.  This runs that same bounded wait on an mbarrier nothing
 * ever completes, with a budget of budget_us microseconds, on `device`:
 * it returns MOE_ERR_TIMEOUT when the timeout path works.  The device stays
 * usable afterwards.  (No counterpart in the reference, whose kernels have no
 * waits.) */
int moe_selftest_wait_timeout(int device, int32_t budget_us);

/* Page-locked host memory for host-side tensors (the reference's
 * Tensor::Alloc::Pinned, src/tensor.cu:11-29), so moe_forward_host's copies
 * run at full link speed.  Free with moe_host_free. */
int moe_host_alloc(size_t bytes, void** out);
int moe_host_free(void* p);

/* Per-expert row counts [E] of the last forward or route on this handle
 * (synchronises the handle's last stream; after a pipelined
 * moe_forward_host, of its last chunk).  The dispatch histogram of
 * src/model.cu:921-1003. */
int moe_expert_counts(MoeHandle* h, int32_t* counts);

/* Dispatch layout of the last forward (synchronises): for each packed row
 * (rows are grouped by expert, each expert's block starting on a multiple of
 * 128 rows) the source token (-1 for padding rows) and its combine weight.
 * `rows_cap` is the capacity of the two arrays; *rows_out receives the number
 * of packed rows.  Replaces route_place's index (src/model.cu:1009-1030). */
int moe_dispatch_layout(MoeHandle* h, int32_t* row_token, float* row_weight, int32_t rows_cap,
                        int32_t* rows_out, int32_t* expert_offsets /* [E+1] or NULL */);

/* Per-stage device timers, the counterpart of the reference's APS_PROFILE
 * stage timers (src/model.cu:1584-1622, 2052-2058).  When enabled, forward
 * records a CUDA event on its stream at each stage boundary (no host
 * synchronisation; dependent launches are turned off so the events sit
 * between the kernels).  moe_profile_read synchronises on the last event and
 * writes the milliseconds of each stage of the last forward:
 *   [0] router (batches of <= 4 tokens: router, layout and row packing)
 *   [1] dispatch scan  [2] dispatch permute (expert parallel: also the
 *       arrival scan and arrangement)
 *   [3] gate/up grouped GEMM (decode path: decode gate/up kernel)
 *   [4] down grouped GEMM (decode path: decode down kernel)
 *   [5] expert parallel: counts exchange, host plan, payload exchange
 *   [6] expert parallel: return exchange  [7] expert parallel: combine
 * Stages a forward did not run read 0.  Returns the number of stages (8). */
#define MOE_PROFILE_STAGES 8
int moe_profile_enable(MoeHandle* h, int enable);
int moe_profile_read(MoeHandle* h, float* stage_ms, int32_t n);

/* ---------------------------------------------------------------------
 * Expert parallelism (no counterpart in the reference, which runs on one
 * GPU): one process and one GPU per rank, experts placed round-robin
 * (rank r holds experts r, r + G, r + 2G, ...; a skewed router's hot
 * experts land on different ranks), router weights replicated.  Expert e's
 * dispatch position is (e % G) * (E / G) + e / G, so each rank's experts
 * form one contiguous run of positions.  Dispatch and combine cross NVLink
 * as peer stores (MOE_EP_TRANSPORT_P2P) or NCCL point-to-point exchanges
 * (MOE_EP_TRANSPORT_NCCL).  NCCL is loaded at run time (libnccl.so.2);
 * MOE_ERR_NCCL if it is absent.
 * --------------------------------------------------------------------- */

/* The exchange plan of one forward, host only (no GPU needed): from this
 * rank's routed rows per dispatch position `counts` [world * e_local] and the
 * rows each source sends it for its local experts `counts_in`
 * [world][e_local], the rows sent to / received from each rank and their
 * offsets in the (expert-sorted) send and (source-major) receive buffers.
 * send_off / recv_off have world + 1 entries. */
int moe_ep_plan(const int32_t* counts, const int32_t* counts_in, int32_t world, int32_t e_local,
                int64_t* send_rows, int64_t* send_off, int64_t* recv_rows, int64_t* recv_off);

/* 128-byte NCCL unique id for a new group: rank 0 calls this and hands the
 * bytes to every rank by its own means (a store, a broadcast, a file). */
int moe_ep_unique_id(void* id_out);

/* Collective over the group: every rank calls it with the same global
 * config (num_experts a multiple of `world`) and the same id.  `weights`
 * holds pointers for all E experts, in the experts' own order; only this
 * rank's experts (r, r + G, ...) are read, so the others may be any
 * non-null placeholder (host pointers here, device pointers on cfg->device
 * for the _from_device variant). */
int moe_ep_create(const MoeConfig* cfg, const MoeWeightsHost* weights, int rank, int world,
                  const void* nccl_id, MoeHandle** out);
int moe_ep_create_from_device(const MoeConfig* cfg, const MoeWeightsHost* weights, int rank,
                              int world, const void* nccl_id, MoeHandle** out);

/* Collective forward: each rank passes its own T local tokens (T may differ
 * between ranks, and may be 0) and gets its own y.  Synchronises the stream
 * once, after the counts exchange, to size the payload exchange.
 * moe_destroy releases the group's communicator. */
int moe_ep_forward_device(MoeHandle* h, const float* x, float* y, int32_t T, void* stream);

/* Failure of the fused transport.  Every peer wait is bounded
 * (MoeConfig.ep_wait_ms).  A rank whose wait runs out marks itself failed on
 * the device: from then on its kernels store nothing into other GPUs'
 * buffers and raise no flags, and its own waits end at once, so no rank
 * hangs and no late peer's rows are mixed into a later step; the other ranks'
 * waits then run out too.  moe_ep_forward_device enqueues without host
 * synchronisation, so it reports the failure of an earlier step
 * (MOE_ERR_TIMEOUT) once that step has completed on the GPU; moe_ep_check
 * waits for the last forward and reports it at once.  After MOE_ERR_TIMEOUT
 * the handle stays failed: every later forward returns MOE_ERR_TIMEOUT
 * without launching anything, and the group must be destroyed and created
 * again (on every rank).  The NCCL transport reports through NCCL. */
int moe_ep_check(MoeHandle* h);

/* Dispatch that allocates nothing.  No counterpart in the reference: it
 * exists for callers that cannot call cudaMalloc -- code running inside a
 * stream capture that must not touch the allocator, frameworks that own all
 * device memory through their own pool, latency-critical paths that cannot
 * afford an allocation's implicit synchronisation.
 *
 * From routing decisions already on the device (idx / weights [T][top_k],
 * e.g. from moe_route_device) it writes the same packed layout the forward
 * path uses: expert blocks padded to multiples of 128 rows, tokens in
 * ascending order inside each block, row_token = -1 and row_weight = 0 on
 * padding rows, expert_offsets [E+1], counts [E].  All outputs are device
 * buffers; rows_cap must be >= (T * top_k / 128 + num_experts + 1) * 128.
 * Expert indices outside [0, num_experts) are not placed; an expert that one
 * token lists twice gets two rows, in slot order (the router never does
 * this).  T == 0 writes zero counts and offsets.
 *
 * Its only scratch is a fixed 1 MiB array in the library's device memory
 * (MOE_NOALLOC_SCRATCH_BYTES, present on every GPU that loads the library
 * until the process exits), so ceil(T / 32) * num_experts may not exceed
 * 262144; larger calls are rejected with MOE_ERR_INVALID.  The first call on
 * a device looks up that array's address, so make it before any stream
 * capture starts.  All calls on a device share the array: calls whose GPU
 * work can overlap race and must be serialised by the caller.  Enqueued on
 * `stream` with no host synchronisation. */
#define MOE_NOALLOC_SCRATCH_BYTES (1u << 20)
int moe_dispatch_noalloc(const int32_t* idx, const float* weights, int32_t T,
                         int32_t num_experts, int32_t top_k, int32_t* row_token,
                         float* row_weight, int32_t rows_cap, int32_t* expert_offsets,
                         int32_t* counts, void* stream);

/* ---------------------------------------------------------------------
 * Whole-model greedy generation with the MoE layers above: the toy MoE
 * decoder of BASELINE config 4, the counterpart of the reference's
 * PhiTinyMoEModel (include/model.h:8-30): generate (src/model.cu:1575-2058,
 * last-position logits of a batch) and generate_decode (src/model.cu:
 * 2061-2104, greedy argmax, first maximum wins, stop at EOS).
 *
 * Architecture: tied token embeddings; per layer x += o_proj(attn(rope(
 * qkv_proj(rms_norm(x))))) then x += MoE(rms_norm(x)); a final rms_norm and
 * the embedding matrix as the output head.  Multi-head attention (as many KV
 * heads as query heads), causal, scaled by 1/sqrt(head_dim); rotary
 * embedding in the reference's rotate-half form (tensor_ops::apply_rope,
 * src/tensor.cu:191-210), its cos/sin table computed in double.  The MoE is
 * the softmax / top-k / renormalise router with SwiGLU experts.  Unlike the
 * reference's generate_decode, which re-runs the whole prefix per token, the
 * decoder keeps a KV cache, so each new token costs one decode step.
 *
 * The projections and the output head run on the same tcgen05 grouped GEMM
 * as the experts (one group, identity row map); precision as MoeConfig's.
 * Constraints: d_model == n_heads * head_dim, d_model a multiple of 128,
 * head_dim 64 or 128, vocab a multiple of 32; every sequence of a batch has
 * the same length; max_batch * max_seq rows of activations are reserved.
 * --------------------------------------------------------------------- */
typedef struct MoeDecoderConfig {
    int32_t n_layers;
    int32_t d_model;
    int32_t n_heads;
    int32_t head_dim;
    int32_t vocab;
    int32_t num_experts;
    int32_t top_k;
    int32_t d_ff;
    float rms_eps;       /* 1e-5 */
    float rope_base;     /* 10000 */
    int32_t precision;   /* MoePrecision */
    int32_t max_batch;   /* sequences per call */
    int32_t max_seq;     /* prompt + generated tokens per sequence */
    int32_t device;
    int32_t reserved[4];
} MoeDecoderConfig;

/* fp32 nn.Linear-layout weights ([out][in], row-major).  Per-layer entries
 * are arrays of n_layers pointers; expert entries n_layers * num_experts
 * pointers, layer-major.  Host pointers for moe_decoder_create, device
 * pointers (on cfg->device) for moe_decoder_create_from_device; copied and
 * converted, the caller keeps ownership. */
typedef struct MoeDecoderWeights {
    const float* embed;             /* [vocab][d_model]; also the output head */
    const float* final_norm;        /* [d_model] */
    const float* const* attn_norm;  /* [d_model] each */
    const float* const* wq;         /* [d_model][d_model] each */
    const float* const* wk;
    const float* const* wv;
    const float* const* wo;
    const float* const* ffn_norm;   /* [d_model] each */
    const float* const* router;     /* [num_experts][d_model] each */
    const float* const* w1;         /* [d_ff][d_model] each */
    const float* const* w3;         /* [d_ff][d_model] each */
    const float* const* w2;         /* [d_model][d_ff] each */
} MoeDecoderWeights;

typedef struct MoeDecoder MoeDecoder;

/* Defaults of BASELINE config 4 (8 layers, d 2048, 16 x 128 heads, vocab
 * 32000, 16 experts top-2, d_ff 5632, eps 1e-5, RoPE base 10000), BF16,
 * batch 16, 640 positions, device 0. */
void moe_decoder_config_init(MoeDecoderConfig* cfg);
int moe_decoder_create(const MoeDecoderConfig* cfg, const MoeDecoderWeights* w,
                       MoeDecoder** out);
int moe_decoder_create_from_device(const MoeDecoderConfig* cfg, const MoeDecoderWeights* w,
                                   MoeDecoder** out);
void moe_decoder_destroy(MoeDecoder* m);
size_t moe_decoder_device_bytes(const MoeDecoder* m);

/* Prefill (PhiTinyMoEModel::generate): tokens [B][S] (host int32) fill the
 * KV cache from position 0 and give the last position's logits [B][vocab]
 * and greedy next ids [B] (host; either may be NULL).  Synchronises. */
int moe_decoder_prefill(MoeDecoder* m, const int32_t* tokens, int32_t B, int32_t S,
                        float* logits, int32_t* next_ids);
/* One decode step after a prefill or an earlier step: tokens [B] (host) go
 * in at the next position of every sequence; logits [B][vocab] and the
 * greedy next ids [B] come out (host; either may be NULL).  Synchronises.
 * MOE_ERR_INVALID past max_seq. */
int moe_decoder_decode_step(MoeDecoder* m, const int32_t* tokens, float* logits,
                            int32_t* next_ids);
/* Greedy generation (PhiTinyMoEModel::generate_decode): prefill the prompt
 * [B][S], then max_new_tokens greedy tokens per sequence.  ids [B][n] (host)
 * receive the generated tokens; logits [B][n][vocab] (host, may be NULL) the
 * logits each token was chosen from.  A sequence that emits eos_id (pass -1
 * for none) stops there: its later ids are -1 and its later logits 0.
 * Decode steps keep the tokens on the device; one synchronisation at the
 * end. */
int moe_decoder_generate(MoeDecoder* m, const int32_t* prompt, int32_t B, int32_t S,
                         int32_t max_new_tokens, int32_t eos_id, float* logits, int32_t* ids);
/* Device time (CUDA events on the decoder's stream) of the last
 * moe_decoder_generate: the prefill (through the first token's argmax) and
 * all decode steps. */
int moe_decoder_last_timing(const MoeDecoder* m, float* prefill_ms, float* decode_ms);
/* Fused batch-1 decode step (no counterpart in the reference, whose
 * generate_decode re-runs the whole prefix per token, src/model.cu:2061-2104):
 * with one sequence in BF16 precision a decode step can run as ONE
 * cooperative launch over every layer and the output head, grid-wide
 * barriers between its phases, instead of about ten kernels per layer; its
 * logits are bit-identical to the kernel chain's.  Off by default (at config
 * 4 the chain measured 0.74 ms per step, the fused step 0.99 ms).
 * enable = 1 selects the fused step, 0 the chain; MOE_ERR_UNSUPPORTED when
 * enabling a configuration it does not cover (FP32 precision, more experts
 * than SMs, d_model > 8192). */
int moe_decoder_set_fused_step(MoeDecoder* m, int32_t enable);
/* 1 if batch-1 decode steps run the fused step, else 0 (or a null m). */
int moe_decoder_fused_step_active(const MoeDecoder* m);

#ifdef __cplusplus
}
#endif
#endif /* MOE_B200_H */
