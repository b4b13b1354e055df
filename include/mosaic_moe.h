/*
 * mosaic_moe.h — C ABI of the B200 (sm_100a) MoE-layer hot path.
 *
 * Plain pointers and sizes only.  Every pointer argument is a DEVICE pointer
 * unless stated otherwise; every call is asynchronous on the given stream,
 * performs no host synchronisation and allocates nothing (the caller passes
 * outputs and a workspace sized by the matching *_workspace_bytes call), so
 * a whole layer can be captured in a CUDA graph.  The exceptions are the
 * one-time set-up calls of the peer-memory exchange (mosaic_ep_region_alloc /
 * _open / _close / _free), which allocate, map and synchronise.  Shapes, alignment and
 * ranges are checked on the host before anything is launched; a failed check
 * returns a MOSAIC_ERR_* code and launches nothing.  Errors found on the
 * device (an expert id out of range, a pipeline wait that timed out) are
 * recorded in an error word inside the workspace: read it with
 * mosaic_read_error().
 *
 * Reference interfaces replaced (paths inside fazin-ahamed/Mosaic):
 *   mosaic_router            <- mosaicvm/model/layers.py:118-150 (Router.forward) with the
 *                               sigmoid score of .mosaicvm/source/inference_model.py:569-589 (Gate)
 *   mosaic_router_ext        <- the same plus the other score functions
 *                               (layers.py:110-115 _router_scores: sqrt(softplus); Gate: softmax)
 *                               and hash routing (layers.py:153-197 HashRouter.forward; Gate's
 *                               tid2eid branch, inference_model.py:581-582)
 *   mosaic_layout_assignments<- mosaicvm/kernels/moe_layout.py:8-27 (layout_assignments)
 *   mosaic_emit_tiles        <- mosaicvm/kernels/w4a16_grouped.py:151-169 (emit_tiles)
 *   mosaic_act_quant         <- mosaicvm/kernels/fp4_source.py:110-129 (act_quant_ref)
 *   mosaic_pack_mxfp4        <- mosaicvm/kernels/fp4_source.py:35-64 (pack_mxfp4_nk)
 *   mosaic_prepack_scales    <- mosaicvm/kernels/qpa_mma.py:577-613 (prepack_expert_bank_qpa:
 *                               an invertible re-layout of the expert bank, scales only here)
 *   mosaic_moe_routed        <- mosaicvm/kernels/exact_moe.py:12-19 (exact_moe) /
 *                               mosaicvm/kernels/qpa_mma.py:681-784 (fused_moe_qpa)
 *   mosaic_expert_gemm_gu /  <- mosaicvm/kernels/qpa_mma.py:750-772 (fused_moe_qpa's gate/up and
 *   mosaic_expert_gemm_down     down calls of _run_two_queues, :787-830)
 *   mosaic_moe_forward       <- mosaicvm/model/layers.py:284-303 (MoELayer.forward)
 *   mosaic_moe_forward_ext   <- the same with mosaic_router_ext's routing, which with hash
 *                               routing is layers.py:394-405 (HashMoELayer.forward)
 *   mosaic_hc_pre_norm       <- mosaicvm/model/layers.py:258-267 (HyperConnections.pre, with
 *                               hc_split_sinkhorn :222-234) + :19-29 (RMSNorm, the block's
 *                               ffn_norm, :431-433) + fp4_source.py:110-129 (act_quant_ref)
 *   mosaic_hc_post           <- mosaicvm/model/layers.py:269-271 (HyperConnections.post)
 *   mosaic_rms_norm          <- mosaicvm/model/layers.py:19-29 (RMSNorm.forward)
 *   mosaic_ep_*              <- .mosaicvm/source/inference_model.py:614-650 (MoE.forward,
 *                               expert-sharded; all_reduce replaced by all-to-all)
 */
#ifndef MOSAIC_MOE_H_
#define MOSAIC_MOE_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define MOSAIC_API __attribute__((visibility("default")))
#else
#define MOSAIC_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Same object as cudaStream_t / CUstream; NULL is the legacy default stream. */
typedef struct CUstream_st* mosaic_stream_t;

enum mosaic_status {
  MOSAIC_OK = 0,
  MOSAIC_ERR_SHAPE = 1,       /* dimension contract violated (ValueError in the reference) */
  MOSAIC_ERR_DTYPE = 2,       /* unsupported number format */
  MOSAIC_ERR_ALIGN = 3,       /* pointer alignment contract violated */
  MOSAIC_ERR_RANGE = 4,       /* value out of range (expert id, scale byte) */
  MOSAIC_ERR_CUDA = 5,        /* CUDA runtime / driver error */
  MOSAIC_ERR_TIMEOUT = 6,     /* a device pipeline wait gave up (kernel returned early) */
  MOSAIC_ERR_UNSUPPORTED = 7, /* configuration outside what the kernels implement */
  MOSAIC_ERR_WORKSPACE = 8    /* workspace too small */
};

/* Activation formats of the expert GEMMs.
 * MOSAIC_ACT_BF16: bf16 activations (decode).  Each bf16 value is carried
 *   into the block-scaled MMA as the sum of two E4M3 values with their own
 *   per-32 power-of-two scales (hi + lo), which represents it to ~2^-8.
 * MOSAIC_ACT_FP8: the reference's source semantics — act_quant_ref (E4M3,
 *   power-of-two scale per 1x128 block) on the expert inputs, bf16 outputs
 *   of every expert linear. */
enum mosaic_act_mode { MOSAIC_ACT_BF16 = 0, MOSAIC_ACT_FP8 = 1 };

typedef struct mosaic_moe_dims {
  int32_t tokens;         /* T: rows of x */
  int32_t hidden;         /* H: multiple of 256 */
  int32_t inter;          /* I: moe_intermediate_size, multiple of 128 */
  int32_t n_experts;      /* E routed experts, 1..256 */
  int32_t top_k;          /* 1..8, <= E */
  int32_t n_group;        /* router groups (1 = no group limit); divides E */
  int32_t topk_group;     /* groups kept per token */
  int32_t act_mode;       /* enum mosaic_act_mode */
  int32_t norm_topk_prob; /* 1: weights /= sum(weights).clamp_min(1e-9) */
  int32_t has_shared;     /* 1: the bank holds the shared expert as expert E and y includes it */
  float route_scale;      /* routed_scaling_factor */
  float swiglu_limit;     /* 0 = no clamp; else gate <= limit, |up| <= limit */
} mosaic_moe_dims;

/* Expert bank (device memory).  n_bank = E + has_shared; the shared expert,
 * when present, is the last one.  The reference layout
 * (mosaicvm/kernels/exact_moe.py:12: packed_gate_up uint8 [E, 2I, H/2], gate
 * rows then up rows, low nibble = even K; packed_down [E, H, I/2]; E8M0
 * scales [E, rows, K/32]) is re-laid out once, invertibly (the role of
 * mosaicvm/kernels/qpa_mma.py:577-613 prepack_expert_bank_qpa): codes by
 * mosaic_repack_weights into contiguous 8 KB tiles, scales by
 * mosaic_prepack_scales into the 512-byte chunks the MMA reads. */
typedef struct mosaic_expert_bank {
  const uint8_t* gu_tiled;  /* [n_bank][I/128][H/128][2][128][64]: mosaic_repack_weights(halves=2), 32-B aligned */
  const uint8_t* gu_sf;     /* [n_bank][I/128][H/128][2][512]: mosaic_prepack_scales(halves=2) */
  const uint8_t* dn_tiled;  /* [n_bank][H/256][I/128][2][128][64]: mosaic_repack_weights(halves=2), 32-B aligned */
  const uint8_t* dn_sf;     /* [n_bank][H/256][I/128][2][512]: mosaic_prepack_scales(halves=2) */
} mosaic_expert_bank;

MOSAIC_API int mosaic_version(void);
MOSAIC_API const char* mosaic_status_string(int status);
/* Number of SMs of the current device (0 when no device). */
MOSAIC_API int mosaic_device_sm_count(void);

/* Router: logits = x @ W^T in fp32, s = sigmoid(logits), selection on s + bias
 * (fp32, selection only), optional group limit (sum of the top-2 biased
 * scores per group, keep topk_group groups), top_k in descending order of the
 * biased score, weights gathered from the unbiased s, normalised and scaled.
 * x bf16 [T, H]; weight fp32 [E, H]; bias fp32 [E] (NULL = zeros);
 * weights_out fp32 [T, top_k]; idx_out int64 [T, top_k].
 * Equal biased scores are broken towards the lower expert id.  The
 * workspace's error word (its first 16 bytes) is cleared at the start of
 * each call; read it afterwards with mosaic_read_error. */
MOSAIC_API size_t mosaic_router_workspace_bytes(int32_t T, int32_t H, int32_t E);
MOSAIC_API int mosaic_router(const void* x, const float* weight, const float* bias, int32_t T, int32_t H, int32_t E,
                  int32_t top_k, int32_t n_group, int32_t topk_group, float route_scale, int32_t norm_topk_prob,
                  float* weights_out, int64_t* idx_out, void* workspace, size_t workspace_bytes,
                  mosaic_stream_t stream);

/* Score functions of the router (the reference's scoring_func / score_func). */
enum mosaic_score_func {
  MOSAIC_SCORE_SIGMOID = 0,      /* 1 / (1 + exp(-l))          inference_model.py:573-574 */
  MOSAIC_SCORE_SQRTSOFTPLUS = 1, /* sqrt(softplus(l)), softplus threshold 20   layers.py:110-115 */
  MOSAIC_SCORE_SOFTMAX = 2       /* exp(l - max) / sum over the E experts  inference_model.py:571-572 */
};

/* Router variant: score function and hash routing.  NULL = sigmoid top-k. */
typedef struct mosaic_route_ext {
  int32_t score_func;       /* enum mosaic_score_func */
  int32_t hash;             /* 1: expert ids by token id, not by score (HashRouter) */
  int32_t layer_idx;        /* hash without a table: the salt's layer index, >= 0 */
  int32_t reserved;         /* 0 */
  int64_t table_rows;       /* rows of tid2eid (the vocabulary size), >= 1 */
  const int32_t* tid2eid;   /* hash table int32 [table_rows, top_k] (device), row token % table_rows
                               (floor modulo); NULL with hash = 1: the salted hash, top_k 1 */
  const int64_t* token_ids; /* int64 [T] (device); NULL = 0..T-1 */
} mosaic_route_ext;

/* mosaic_router with a variant (ext NULL: identical to mosaic_router).
 * Score s = score_func(logits); without hash the selection is as in
 * mosaic_router on s + bias.  With hash the ids of token t are row
 * token_ids[t] mod table_rows of tid2eid in table order (an id outside
 * [0, E) sets MOSAIC_ERR_RANGE in the error word and reads as 0), the group
 * limit and bias play no part, and the weights are s gathered at those ids,
 * normalised when norm_topk_prob and times route_scale (the reference
 * normalises unless the score is softmax: pass norm_topk_prob accordingly).
 * Without a table (tid2eid NULL) top_k must be 1, no logits are computed,
 * weight = route_scale and id = hashed mod E with
 * salt = layer_idx * 2654435761 mod 2^31 and
 * hashed = ((int32(token) + salt) * 2654435761) mod 2^31 in int32 tensor
 * arithmetic (layers.py:180-184 as torch evaluates it: wrapping sum and
 * product, the literal 2^31 read as -2^31, floor modulo).  x and weight may
 * be NULL in that case. */
MOSAIC_API int mosaic_router_ext(const mosaic_route_ext* ext, const void* x, const float* weight, const float* bias,
                                 int32_t T, int32_t H, int32_t E, int32_t top_k, int32_t n_group,
                                 int32_t topk_group, float route_scale, int32_t norm_topk_prob, float* weights_out,
                                 int64_t* idx_out, void* workspace, size_t workspace_bytes, mosaic_stream_t stream);

/* Size of the fixed device scratch of mosaic_router_noalloc (32 MiB). */
#define MOSAIC_ROUTER_NOALLOC_SCRATCH_BYTES (32u << 20)

/* mosaic_router without a caller workspace; it has no counterpart in the
 * reference (whose Router.forward allocates through torch).  The split-K
 * logit partials live in a file-scope device array of
 * MOSAIC_ROUTER_NOALLOC_SCRATCH_BYTES, so the call allocates and frees no
 * device memory (no cudaMalloc/cudaFree, no torch allocator); results are
 * bit-identical to mosaic_router on the same inputs.  Inputs whose partials
 * need more than the scratch (mosaic_router_workspace_bytes(T, H, E) >
 * MOSAIC_ROUTER_NOALLOC_SCRATCH_BYTES, e.g. T = 32768, H = 7168, E = 256)
 * return MOSAIC_ERR_WORKSPACE without launching.
 * - One scratch per device: calls that overlap on a device (two streams, two
 *   host threads, or two launches in one graph that may run concurrently)
 *   race on it and give undefined results.  Serialise them.
 * - Every call outside stream capture looks up the scratch address
 *   (cudaGetSymbolAddress, which may load the module); a call under capture
 *   uses the address its device's last uncaptured call found, so the first
 *   call on each device must come before any stream capture.
 * - Device errors (a non-finite score, a pipeline wait of the tensor-core
 *   logits that ran out) go to the scratch's error word, which each call
 *   clears first and which this entry point does not report: its outputs
 *   are then undefined.  Use mosaic_router with mosaic_read_error where that
 *   check is needed. */
MOSAIC_API int mosaic_router_noalloc(const void* x, const float* weight, const float* bias, int32_t T, int32_t H,
                                     int32_t E, int32_t top_k, int32_t n_group, int32_t topk_group,
                                     float route_scale, int32_t norm_topk_prob, float* weights_out,
                                     int64_t* idx_out, mosaic_stream_t stream);

/* ids int64 [A] -> sorted_ids int64 [A], perm int64 [A] (stable: ascending
 * flat index inside each expert segment), offsets int32 [E+1], counts int32 [E].
 * One CTA (histogram, prefix scan, stable scatter in 1024-id chunks); A <= 1<<20.
 * The MoE layer's own layout (inside mosaic_moe_forward) uses a multi-CTA
 * count / scan / rank pass above 1024 assignments instead. */
MOSAIC_API int mosaic_layout_assignments(const int64_t* expert_ids, int32_t A, int32_t E, int64_t* sorted_ids,
                              int64_t* perm, int32_t* offsets, int32_t* counts, mosaic_stream_t stream);

/* counts int32 [E] -> tiles (expert_index, m_start, tile_rows) int32 [max_tiles]
 * in expert order and n_tiles int32 [1]; tiles beyond max_tiles are dropped
 * and flagged by n_tiles > max_tiles. */
MOSAIC_API int mosaic_emit_tiles(const int32_t* counts, int32_t E, int32_t block_m, int32_t max_tiles,
                      int32_t* expert_index, int32_t* m_start, int32_t* n_tiles, int32_t* tile_rows,
                      mosaic_stream_t stream);

/* act_quant_ref: x bf16 [M, K] -> q e4m3fn bytes [M, K], scale fp32 [M, K/128]. */
MOSAIC_API int mosaic_act_quant(const void* x, int32_t M, int32_t K, uint8_t* q, float* scale, mosaic_stream_t stream);

/* pack_mxfp4_nk: w fp32 [N, K] -> packed uint8 [N, K/2], E8M0 scale uint8 [N, K/32]
 * (FLOOR E8M0, RNE E2M1 with saturation; bit-identical to the reference packer). */
MOSAIC_API int mosaic_pack_mxfp4(const float* w, int32_t N, int32_t K, uint8_t* packed, uint8_t* scale,
                      mosaic_stream_t stream);

/* Re-lay packed E2M1 codes [n_mats][rows][K/2] (the reference layout) into
 * 8 KB tiles of 128 rows x 128 values, [n_mats][row block][K/128][halves][128][64].
 * halves = 2 splits the rows into two halves (gate rows, up rows) and puts the
 * two tiles of the same row block and K-tile next to each other; halves = 1 is
 * plain.  rows % (128 * halves) == 0, K % 128 == 0, 16-B aligned pointers. */
MOSAIC_API int mosaic_repack_weights(const uint8_t* packed, int32_t n_mats, int32_t rows, int32_t K, int32_t halves,
                                     uint8_t* tiled, mosaic_stream_t stream);

/* Re-lay E8M0 scales [n_mats][rows][K/32] into the chunks the block-scaled MMA
 * consumes, in the same tile order as mosaic_repack_weights:
 * [n_mats][row block][K/128][halves][512], byte (r%32)*16 + ((r%128)/32)*4 + kb
 * of a chunk holding row r, K32 block kb.  rows % (128 * halves) == 0, K % 128 == 0. */
MOSAIC_API int mosaic_prepack_scales(const uint8_t* scale, int32_t n_mats, int32_t rows, int32_t K, int32_t halves,
                                     uint8_t* sf_chunks, mosaic_stream_t stream);

/* The step in front of the MoE in a V4 block (layers.py:428-433): the
 * hyper-connection pre-mix of the hc residual copies, then the ffn RMSNorm,
 * fused; optionally also act_quant_ref of the result (the FP8 MoE input).
 *   x           bf16 [T, hc, D] (the block's residual stream)
 *   fn          fp32 [(2+hc)*hc, hc*D]; base fp32 [(2+hc)*hc]; scale fp32 [3]
 *   norm_weight fp32 [D] (RMSNorm weight), or NULL for the pre-mix alone
 *               (HyperConnections.pre); norm_eps both for the rsqrt of the
 *               pre-mix and for the RMSNorm (both use rms_norm_eps); hc_eps the
 *               Sinkhorn epsilon; sinkhorn_iters >= 1
 *   y           bf16 [T, D] = RMSNorm(sum_m pre_m * x_m), the MoE input
 *   post        fp32 [T, hc], comb fp32 [T, hc, hc]: for mosaic_hc_post
 *   q, q_scale  E4M3 [T, D] and fp32 [T, D/128] = act_quant_ref(y), or both NULL
 * hc 1..4; D a multiple of 128, at most 16384 (MOSAIC_ERR_UNSUPPORTED above:
 * the pre-mix row is held in registers); x, y, q 16-byte aligned; fn,
 * norm_weight too.  The workspace (256-B aligned,
 * mosaic_hc_pre_norm_workspace_bytes) holds the error word
 * (mosaic_read_error), the split-K partials of the mixing products, fn split
 * into three bf16 parts for the tensor cores and the tokens' pre-mix weights. */
MOSAIC_API size_t mosaic_hc_pre_norm_workspace_bytes(int32_t T, int32_t D, int32_t hc);
MOSAIC_API int mosaic_hc_pre_norm(const void* x, const float* fn, const float* base, const float* scale,
                                  const float* norm_weight, int32_t T, int32_t D, int32_t hc, int32_t sinkhorn_iters,
                                  float hc_eps, float norm_eps, void* y, float* post, float* comb, uint8_t* q,
                                  float* q_scale, void* workspace, size_t workspace_bytes, mosaic_stream_t stream);

/* RMSNorm on its own, mosaicvm/model/layers.py:19-29 (RMSNorm.forward):
 * y[t] = bf16(x[t] * (1 / sqrt(mean(x[t]^2) + eps)) * weight), all in fp32.
 *   x, y        bf16 [T, D], 16-byte aligned; D % 8 == 0, D <= MOSAIC_RMS_NORM_MAX_D
 *   weight      fp32 [D], 16-byte aligned
 *   q, q_scale  E4M3 [T, D] and fp32 [T, D/128] = act_quant_ref(y) (the FP8 MoE
 *               input; D % 128 == 0), or both NULL
 * One row per CTA, read from HBM once; no workspace. */
#define MOSAIC_RMS_NORM_MAX_D 65536
MOSAIC_API int mosaic_rms_norm(const void* x, const float* weight, int32_t T, int32_t D, float eps, void* y,
                               uint8_t* q, float* q_scale, mosaic_stream_t stream);

/* The step behind the MoE: out[t, m] = post[t, m] * y[t] + sum_n comb[t, m, n] * residual[t, n]
 * (fp32, rounded to bf16); y bf16 [T, D] (the MoE output), residual and out bf16 [T, hc, D]. */
MOSAIC_API int mosaic_hc_post(const void* y, const void* residual, const float* post, const float* comb, int32_t T,
                              int32_t D, int32_t hc, void* out, mosaic_stream_t stream);

/* Workspace for mosaic_moe_forward / mosaic_moe_routed (256-B aligned pointer). */
MOSAIC_API size_t mosaic_moe_workspace_bytes(const mosaic_moe_dims* dims);

/* Full MoE layer: router -> layout -> expert gate/up (+SwiGLU, x route weight)
 * -> down -> ordered combine (+ shared expert).  x, y bf16 [T, H].
 * weights_out fp32 [T, top_k] and idx_out int64 [T, top_k] receive the routing. */
MOSAIC_API int mosaic_moe_forward(const mosaic_moe_dims* dims, const void* x, const float* router_weight,
                       const float* router_bias, const mosaic_expert_bank* bank, void* y, float* weights_out,
                       int64_t* idx_out, void* workspace, size_t workspace_bytes, mosaic_stream_t stream);

/* mosaic_moe_forward with the routing of mosaic_router_ext (ext NULL:
 * identical to mosaic_moe_forward).  With hash routing and a table this is
 * HashMoELayer.forward (layers.py:394-405): ids from tid2eid, weights from the
 * router scores; router_bias is ignored. */
MOSAIC_API int mosaic_moe_forward_ext(const mosaic_moe_dims* dims, const mosaic_route_ext* ext, const void* x,
                                      const float* router_weight, const float* router_bias,
                                      const mosaic_expert_bank* bank, void* y, float* weights_out, int64_t* idx_out,
                                      void* workspace, size_t workspace_bytes, mosaic_stream_t stream);

/* mosaic_moe_forward that also records caller-created CUDA events
 * (cudaEvent_t handles, any slot may be NULL) on the stream at the stage
 * boundaries: [0] start, [1] after the router, [2] after the layout, [3]
 * after quantisation, [4] after the gate/up GEMM, [5] after the down GEMM,
 * [6] after the combine.  For per-kernel timing. */
MOSAIC_API int mosaic_moe_forward_profiled(const mosaic_moe_dims* dims, const void* x, const float* router_weight,
                                           const float* router_bias, const mosaic_expert_bank* bank, void* y,
                                           float* weights_out, int64_t* idx_out, void* workspace,
                                           size_t workspace_bytes, mosaic_stream_t stream,
                                           void* const* stage_events);

/* Routed experts only, routing given (exact_moe contract): x bf16 [T, H];
 * expert_ids int64 [T, top_k]; expert_weights fp32 [T, top_k] (NULL = 1.0);
 * y bf16 [T, H].  dims->has_shared selects whether the bank's last expert
 * (the shared one) is added too. */
MOSAIC_API int mosaic_moe_routed(const mosaic_moe_dims* dims, const void* x, const int64_t* expert_ids,
                      const float* expert_weights, const mosaic_expert_bank* bank, void* y, void* workspace,
                      size_t workspace_bytes, mosaic_stream_t stream);

/* mosaic_moe_routed over an expert cache: the weights and scales of logical
 * expert e (0..n_experts-1, and n_experts = the shared expert when has_shared)
 * are bank entry expert_slot[e] of a bank of bank_slots entries (int32 device
 * table of n_experts + has_shared entries; an entry outside [0, bank_slots)
 * records MOSAIC_ERR_RANGE and reads entry 0).  Everything else uses the
 * logical ids, so the result equals mosaic_moe_routed on a bank that holds the
 * same experts in logical order.  Replaces the per-selected-expert loading of
 * the reference's streaming forward (mosaicvm/runtime/streaming_model.py:209-257,
 * runtime/loader.py:48-71 ExpertLRU) with a device-resident cache. */
MOSAIC_API int mosaic_moe_routed_slots(const mosaic_moe_dims* dims, const void* x, const int64_t* expert_ids,
                                       const float* expert_weights, const mosaic_expert_bank* bank,
                                       const int32_t* expert_slot, int32_t bank_slots, void* y, void* workspace,
                                       size_t workspace_bytes, mosaic_stream_t stream);

/* mosaic_moe_routed in two calls, gate/up then down, in the order the
 * reference runs its grouped kernels (_run_two_queues("gu") then
 * _run_two_queues("down"), mosaicvm/kernels/qpa_mma.py:787-830, inside
 * fused_moe_qpa, qpa_mma.py:681-784).  Same dims, bank and arguments as
 * mosaic_moe_routed; workspace: mosaic_moe_workspace_bytes(dims), shared by
 * the two calls.
 * mosaic_expert_gemm_gu: layout of expert_ids / expert_weights (NULL = 1.0),
 * gather and quantisation of the token rows, then the gate/up GEMM with the
 * clamp, SwiGLU, route weight and act_quant_ref re-quantisation of z fused in
 * its epilogue.  z, the tile list and the row maps stay in the workspace.
 * mosaic_expert_gemm_down: the down GEMM over those z rows, then the ordered
 * combine (ascending expert id in fp32, the shared expert last) into y bf16
 * [T, H].  It must follow a mosaic_expert_gemm_gu call on the same stream
 * with the same dims, bank and workspace, with no other call using that
 * workspace in between.  The two calls give the bytes mosaic_moe_routed
 * gives; the workspace error word keeps what the gate/up call recorded. */
MOSAIC_API int mosaic_expert_gemm_gu(const mosaic_moe_dims* dims, const void* x, const int64_t* expert_ids,
                                     const float* expert_weights, const mosaic_expert_bank* bank, void* workspace,
                                     size_t workspace_bytes, mosaic_stream_t stream);
MOSAIC_API int mosaic_expert_gemm_down(const mosaic_moe_dims* dims, const mosaic_expert_bank* bank, void* y,
                                       void* workspace, size_t workspace_bytes, mosaic_stream_t stream);

/* ---- Expert parallelism -------------------------------------------------
 * Rank d of `world` owns the contiguous experts [d*E/world, (d+1)*E/world)
 * (.mosaicvm/source/inference_model.py:620-627) plus a replica of the shared
 * expert.  One layer step on a rank:
 *   mosaic_router -> mosaic_ep_dispatch -> exchange send rows (all-to-all,
 *   split by dest_counts) -> mosaic_moe_expert_rows on the received rows ->
 *   return the partials (reverse all-to-all) -> mosaic_moe_expert_rows for the
 *   shared expert on the local tokens -> mosaic_ep_combine.
 * The exchange is the caller's (NCCL all_to_all in mosaic_b200/ep.py).
 * Because send rows are sorted by expert id and come back in the order they
 * were sent, the combine sums each token's partials in ascending expert id,
 * exactly as mosaic_moe_forward does: the layer output is bit-identical to
 * the single-GPU layer on the same tokens.
 *
 * Send row (MOSAIC_EP_ROW_BYTES(H) bytes, 16-B aligned): H bf16 token values,
 * then int32 {local expert id, route weight (fp32 bits), source token, dest}. */
#define MOSAIC_EP_ROW_BYTES(H) ((size_t)(H) * 2u + 16u)
/* E4M3 exchange row (MOSAIC_ACT_FP8 layers over the peer-memory exchange with
 * row_e4m3 = 1): the token row quantised as the layer quantises it
 * (act_quant_ref: per 128 values a power-of-two scale, E4M3 codes), H code
 * bytes, then the H/128 biased scale exponents (uint8, 2^(e-127)) padded with
 * zeros to a multiple of 16 bytes, then the same 16-byte tail. */
#define MOSAIC_EP_ROW_BYTES_E4M3(H) ((size_t)(H) + ((((size_t)(H) / 128u) + 15u) & ~(size_t)15u) + 16u)
/* E4M3 unit row (row_e4m3 = 1 with unit_slots = K > 0): one row per (token,
 * owning rank) instead of one per assignment.  The E4M3 row above, whose
 * 16-byte tail becomes a header {slots used, source token, 0, 0}, then K
 * 16-byte slots {local expert id (-1: unused), route weight (fp32 bits),
 * return position (the assignment's row in the source's return buffer), 0}. */
#define MOSAIC_EP_ROW_BYTES_E4M3_UNITS(H, K) (MOSAIC_EP_ROW_BYTES_E4M3(H) + 16u * (size_t)(K))

/* Layout + gather of one rank's assignments.  dims: the layer (tokens = this
 * rank's T, n_experts = global E, E % world == 0).  idx int64 [T, top_k],
 * weights fp32 [T, top_k] (NULL = 1.0); send_rows [T*top_k] rows in expert
 * order (rank-major); dest_counts int32 [world] = rows for each rank.
 * workspace: mosaic_moe_workspace_bytes(dims); keep it for mosaic_ep_combine.
 * Replaces the dispatch half of MoE.forward (inference_model.py:634-650). */
MOSAIC_API int mosaic_ep_dispatch(const mosaic_moe_dims* dims, int32_t world, const void* x, const int64_t* idx,
                                  const float* weights, void* send_rows, int32_t* dest_counts, void* workspace,
                                  size_t workspace_bytes, mosaic_stream_t stream);

/* Per-row expert pass: row r of x_rows (bf16, row stride ldx elements, first
 * H used) goes through expert ids[r * meta_stride] of the bank with route
 * weight weights[r * meta_stride] (weight before down, as in the layer);
 * ids NULL = every row uses default_id, weights NULL = 1.0.  dims: n_experts =
 * routed experts in this bank (<= 256), has_shared = 1 when the bank's last
 * expert (id n_experts) is the shared one; tokens, top_k and the router
 * fields are ignored.  partials [rows, H] in input row order: fp32 in
 * MOSAIC_ACT_BF16 mode, bf16 in MOSAIC_ACT_FP8 mode (what the layer's combine
 * consumes).  rows == 0 is a no-op.  Ids out of range are recorded as
 * MOSAIC_ERR_RANGE in the workspace error word. */
MOSAIC_API size_t mosaic_moe_expert_rows_workspace_bytes(const mosaic_moe_dims* dims, int32_t max_rows);
MOSAIC_API int mosaic_moe_expert_rows(const mosaic_moe_dims* dims, int32_t rows, const void* x_rows, int32_t ldx,
                                      const int32_t* ids, const float* weights, int32_t meta_stride,
                                      int32_t default_id, const mosaic_expert_bank* bank, void* partials,
                                      void* workspace, size_t workspace_bytes, mosaic_stream_t stream);

/* Ordered combine of one rank's returned partials: partials [T*top_k (+ T
 * when dims->has_shared), H] — rows [0, T*top_k) in send-row order, rows
 * [T*top_k, T*top_k + T) the shared expert's partials of the local tokens —
 * same dtype as mosaic_moe_expert_rows writes.  workspace / dims: those of the
 * matching mosaic_ep_dispatch.  y bf16 [T, H]. */
MOSAIC_API int mosaic_ep_combine(const mosaic_moe_dims* dims, const void* partials, const void* workspace, void* y,
                                 mosaic_stream_t stream);

/* ---- Device-driven exchange over NVLink peer memory ----------------------
 * The same dispatch / return steps without host synchronisation, so a whole
 * EP layer step can be captured in a CUDA graph.  Every rank owns one exchange
 * region (mosaic_ep_region_bytes), allocated with mosaic_ep_region_alloc; the
 * 64-byte IPC handles are shared between the ranks over any host channel and
 * opened with mosaic_ep_region_open (plain CUDA IPC mappings of ordinary
 * device memory; no multicast objects).  A region holds: the error word
 * (first 4 bytes, read with mosaic_read_error), per-source flags stamped with
 * a per-step epoch, the world x world row-count matrix, the receive rows and
 * the return partials.  Flags use release / acquire at system scope; every
 * wait is bounded (~2 s) and records MOSAIC_ERR_TIMEOUT in the region.
 * Steps:
 *   mosaic_ep_exchange_rows: publish dest_counts to every rank, wait for all
 *     counts, write this rank's send rows into the owners' receive buffers
 *     (rows from source s after those of sources < s), wait until every
 *     source's rows have landed here.  The received row count is left in the
 *     region (mosaic_ep_region_view) for mosaic_moe_expert_rows' rows_dev.
 *   mosaic_ep_return_partials: write the partial of every received row back
 *     into its source's return buffer at the row's send position, wait for
 *     every owner's partials to land here.  The return buffer then holds the
 *     rows mosaic_ep_combine reads (the caller puts the shared expert's
 *     partials at rows [T*top_k, T*top_k + T)).
 * All ranks must run the same steps in the same order. */
#define MOSAIC_EP_MAX_WORLD 8

typedef struct mosaic_ep_peers {
  int32_t world;          /* ranks, 1..MOSAIC_EP_MAX_WORLD */
  int32_t rank;           /* this rank */
  int32_t max_recv_rows;  /* receive capacity: world * T_max * min(top_k, E / world) covers any routing */
  int32_t max_send_rows;  /* T_max * top_k */
  int32_t max_tokens;     /* T_max (shared-expert rows of the return buffer) */
  int32_t hidden;         /* H */
  int32_t partial_f32;    /* 1: fp32 partials (MOSAIC_ACT_BF16), 0: bf16 (MOSAIC_ACT_FP8) */
  int32_t wait_us;        /* budget of each device-side wait on a peer's flag, in microseconds
                             (0: about 2 s); a wait that runs out records MOSAIC_ERR_TIMEOUT in
                             this rank's region and the kernel returns */
  int32_t row_e4m3;       /* 1: the exchange carries E4M3 rows (MOSAIC_EP_ROW_BYTES_E4M3; needs
                             partial_f32 = 0 and H <= 16384), 0: bf16 rows (MOSAIC_EP_ROW_BYTES) */
  int32_t unit_slots;     /* 0: a row per assignment; K in 1..8 (with row_e4m3 = 1): a row per
                             (token, owning rank) with K slots (K >= min(top_k, experts per rank);
                             MOSAIC_EP_ROW_BYTES_E4M3_UNITS), max_recv_rows counting such rows
                             (world * T_max covers any routing) */
  void* regions[MOSAIC_EP_MAX_WORLD];  /* rank r's region as mapped in this process (own at [rank]) */
} mosaic_ep_peers;

MOSAIC_API size_t mosaic_ep_region_bytes(const mosaic_ep_peers* peers);
MOSAIC_API int mosaic_ep_region_alloc(size_t bytes, void** region, uint8_t* ipc_handle64);
MOSAIC_API int mosaic_ep_region_open(const uint8_t* ipc_handle64, void** peer_region);
MOSAIC_API int mosaic_ep_region_close(void* peer_region);
MOSAIC_API int mosaic_ep_region_free(void* region);
/* Pointers into this rank's own region: receive rows [max_recv_rows][row bytes] (MOSAIC_EP_ROW_BYTES(H),
 * or MOSAIC_EP_ROW_BYTES_E4M3(H) with row_e4m3),
 * the device int32 received-row count, and the return buffer
 * [max_send_rows + max_tokens][H] (fp32 or bf16). */
MOSAIC_API int mosaic_ep_region_view(const mosaic_ep_peers* peers, void** recv_rows, int32_t** recv_count,
                                     void** ret_partials);
MOSAIC_API int mosaic_ep_exchange_rows(const mosaic_ep_peers* peers, const void* send_rows, const int32_t* dest_counts,
                                       mosaic_stream_t stream);
MOSAIC_API int mosaic_ep_return_partials(const mosaic_ep_peers* peers, const void* partials, mosaic_stream_t stream);
/* Dispatch fused with the exchange, for MOSAIC_ACT_FP8 layers with
 * peers->row_e4m3 = 1: the layout of mosaic_ep_dispatch, every token row
 * quantised once (act_quant_ref, as the single-GPU layer does) into scratch
 * rows of the workspace, the count exchange, then each assignment's E4M3 row
 * copied straight into its owner's receive row -- no send buffer, half the
 * NVLink bytes of bf16 rows -- and the wait until every source's rows have
 * landed here.  Replaces mosaic_ep_dispatch +
 * mosaic_ep_exchange_rows; the rows received are what mosaic_ep_dispatch
 * would have sent, quantised.  dims: the layer (tokens = this rank's T <=
 * peers->max_tokens, n_experts = global E, hidden = peers->hidden); idx /
 * weights as for mosaic_ep_dispatch; workspace: mosaic_moe_workspace_bytes(dims),
 * kept for mosaic_ep_combine.  With peers->unit_slots > 0 a token's row goes
 * once to each rank that owns one of its experts, carrying those experts'
 * ids, weights and return positions (at most min(top_k, E/world) slots; at
 * 8 ranks and groups aligned with ranks, at most topk_group rows per token
 * instead of top_k). */
MOSAIC_API int mosaic_ep_dispatch_exchange(const mosaic_moe_dims* dims, const mosaic_ep_peers* peers, const void* x,
                                           const int64_t* idx, const float* weights, void* workspace,
                                           size_t workspace_bytes, mosaic_stream_t stream);
/* The expert pass on this rank's received rows with the return fused in: the
 * down GEMM's epilogue stores every partial straight into its source rank's
 * return buffer (NVLink stores overlapping the GEMM), then every source's
 * return flag is stamped and this rank waits for its own.  Replaces
 * mosaic_moe_expert_rows_dev + mosaic_ep_return_partials.  dims as for
 * mosaic_moe_expert_rows (n_experts = this rank's routed experts); workspace:
 * mosaic_moe_expert_rows_workspace_bytes(dims, peers->max_recv_rows).  With
 * peers->row_e4m3 the received E4M3 rows go into the GEMM's operand planes as
 * they are (no second quantisation; dims->act_mode must be MOSAIC_ACT_FP8). */
/* Workspace of mosaic_ep_expert_rows_return for this exchange (dims as for it):
 * mosaic_moe_expert_rows_workspace_bytes(dims, peers->max_recv_rows) for rows per
 * assignment; with unit rows, room for max_recv_rows * unit_slots assignments. */
MOSAIC_API size_t mosaic_ep_expert_rows_workspace_bytes(const mosaic_moe_dims* dims, const mosaic_ep_peers* peers);
MOSAIC_API int mosaic_ep_expert_rows_return(const mosaic_moe_dims* dims, const mosaic_ep_peers* peers,
                                            const mosaic_expert_bank* bank, void* workspace, size_t workspace_bytes,
                                            mosaic_stream_t stream);
/* mosaic_moe_expert_rows with the row count read on the device from rows_dev
 * (at most max_rows; the workspace is sized for max_rows). */
MOSAIC_API int mosaic_moe_expert_rows_dev(const mosaic_moe_dims* dims, int32_t max_rows, const int32_t* rows_dev,
                                          const void* x_rows, int32_t ldx, const int32_t* ids, const float* weights,
                                          int32_t meta_stride, int32_t default_id, const mosaic_expert_bank* bank,
                                          void* partials, void* workspace, size_t workspace_bytes,
                                          mosaic_stream_t stream);

/* Device error word of a workspace used by mosaic_moe_* (0 = none).
 * Synchronises the stream.  reset != 0 clears it afterwards. */
MOSAIC_API int mosaic_read_error(const void* workspace, int32_t reset, int32_t* code_out, mosaic_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* MOSAIC_MOE_H_ */
