// Internal launch interfaces of the Mosaic B200 MoE kernels (not part of the C ABI).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace mosaic {

// ---- launches
// Inside a PdlScope(true) the chain kernels below are launched with
// programmatic stream serialization: each starts with griddep_wait(), so it
// may be scheduled while its predecessor (a kernel of the same chain) drains.
// Only the single-GPU layer's chain, whose every kernel follows another of its
// kernels in the stream, turns it on.
inline thread_local bool g_pdl_chain = false;
struct PdlScope {
  bool prev;
  explicit PdlScope(bool on) : prev(g_pdl_chain) { g_pdl_chain = on; }
  ~PdlScope() { g_pdl_chain = prev; }
};
template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                            Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = g_pdl_chain ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// ---- grouped block-scaled expert GEMM (gemm_bs.cu)
struct GemmParams {
  int mode;           // 0 = gate/up (+SwiGLU, re-quantise), 1 = down (partials)
                      // a work item is a token tile x a pair of 128-row weight blocks
  int hilo;           // 1: activation rows come as hi and lo E4M3 planes
  int fp8;            // 1: reference FP8 semantics (act_quant per 128, bf16-rounded linears)
  int K;              // reduction length (H for gate/up, I for down)
  int n_blocks;       // block pairs per expert (I/128 gate/up pairs; H/256 down pairs)
  int I, H;
  int R, R_pad;       // packed activation rows (routed + shared) and padded row count
  int shared_expert;  // bank index of the shared expert, or -1
  const int* tiles;   // [max_tiles][3] = (expert, first row, rows)
  const int* n_tiles;
  int max_tiles;
  const uint8_t* x_sft;  // activation scale chunks per token tile: [tile][K/128][512]
  int max_n;             // largest MMA N of the launch (token rows x planes), <= 128
  int brows;             // token rows per activation box (= rows per tile)
  int nbuf;              // TMEM accumulator buffers
  int parities;          // 2: stages alternate between two issuer pairs (own chains); 1: one pair
  const uint8_t* w_sf;   // weight scale chunks [bank][block pair][K/128][half][512]
  const float* row_weight;  // [R] route weight of each packed row
  float swiglu_limit;
  uint8_t* zq;        // gate/up output rows [plane][R_pad][I] (E4M3)
  uint32_t* z_sft;    // their scale chunks per token tile [tile][I/128][128 words]
  void* out;          // down partials [R][H]
  int out_f32;
  const int* out_row; // null: partial of packed row r goes to out row r; else to out row out_row[r]
  // EP return fused into the down epilogue: output row r (after out_row) is a
  // receive row and goes to its source rank's return buffer, found from the
  // geometry in this rank's exchange region header
  int ep_world;       // 0: plain output
  const int* ep_recv_start;
  const int* ep_src_pos;
  const int* ep_row_rank;  // unit rows: packed row r returns to rank ep_row_rank[r], row ep_row_pos[r]
  const int* ep_row_pos;   // (null: from the receive geometry above)
  size_t ep_ret_off;
  uint8_t* ep_regions[MOSAIC_EP_MAX_WORLD];
  // expert offload: the weights of logical expert e are bank entry
  // expert_slot[e] (< bank_slots); null = entry e
  const int* expert_slot;
  int bank_slots;
  int sf_copier;      // 1: the 416-thread kernel, whose warp 12 copies the scale chunks into a
                      // TMEM ring (double-buffered launches); 0: the 384-thread kernel, whose
                      // issuers copy their own (single-buffered wide decode tiles)
  int* err;
};
size_t gemm_smem_bytes(int planes, int brows);
cudaError_t launch_moe_gemm(const CUtensorMap& tmap_w, const CUtensorMap& tmap_x, const GemmParams& p, int grid,
                            cudaStream_t stream);

// ---- router (router.cu)
// Score function and hash routing of one router call (defaults: sigmoid top-k).
struct RouteVariant {
  int score_func = MOSAIC_SCORE_SIGMOID;
  int hash = 0;                        // ids by token id instead of by score
  int32_t salt = 0;                    // table-less hash: layer_idx * 2654435761 mod 2^31
  const int32_t* tid2eid = nullptr;    // [table_rows][top_k]; null with hash = salted hash
  long long table_rows = 0;
  const int64_t* token_ids = nullptr;  // [T]; null = 0..T-1
};
// Split-K factor of the router logits (tensor-core split count where
// router_tc_applies, else the FMA kernels'); the partials are [splits][T][E].
int router_splits(int T, int H, int E, int num_sms);
// Small batches (1 <= T <= 8, H % 64 == 0): logits and top-k in one launch;
// logits [T][E] scratch, arrivals an int the caller zeroes before the launch.
bool router_small_applies(int T, int H, int E);
cudaError_t launch_router_small(const void* x, const float* w, const float* bias, int T, int H, int E, int top_k,
                                int n_group, int topk_group, float route_scale, int norm, float* weights_out,
                                int64_t* idx_out, float* logits, int* arrivals, int* err, cudaStream_t stream,
                                const RouteVariant* variant);
cudaError_t launch_router_topk(const float* partial, int splits, const float* bias, int T, int E, int top_k,
                               int n_group, int topk_group, float route_scale, int norm, float* weights_out,
                               int64_t* idx_out, int* err, cudaStream_t stream, const RouteVariant* variant);
// tensor-core logits (router_tc.cu): x . (hi + mid + lo) with W split into three
// bf16 parts, fp32 partials [splits][T][E].  convert = false: tmap_w maps the
// parts [3E][H] (launch_router_split_w); true: tmap_w maps W fp32 [E][H] and
// the kernel splits it in shared memory.
bool router_tc_applies(int H, int E);
int router_tc_splits(int T, int H, int E, int num_sms);
bool router_tc_convert(int T, int H, int E, int num_sms);
cudaError_t launch_router_split_w(const float* w, int E, int H, void* parts, int num_sms, cudaStream_t stream);
cudaError_t launch_router_logits_tc(const CUtensorMap& tmap_x, const CUtensorMap& tmap_w, bool convert, int T, int H,
                                    int E, int splits, float* out, int* err, cudaStream_t stream);
cudaError_t launch_router(const void* x, const float* w, const float* bias, int T, int H, int E, int top_k,
                          int n_group, int topk_group, float route_scale, int norm, float* weights_out,
                          int64_t* idx_out, float* partial, int splits, int* err, cudaStream_t stream,
                          const RouteVariant* variant = nullptr);

// ---- hyper-connection pre-mix + RMSNorm, post-mix (hc.cu)
struct HcParams {
  const void* x;         // bf16 [T][hc][D]
  const float* fn;       // [(2+hc)*hc][hc*D]
  const float* base;     // [(2+hc)*hc]
  const float* scale;    // [3]
  const float* norm_w;   // [D] RMSNorm weight
  int T, D, hc, iters;
  float hc_eps, norm_eps;
  void* y;               // bf16 [T][D]
  float* post;           // [T][hc]
  float* comb;           // [T][hc][hc]
  uint8_t* q;            // E4M3 [T][D] or null
  float* q_scale;        // [T][D/128]
  float* partial;        // workspace: [splits][T][25] mixing partials (+ sum of squares)
  int splits;
  float* pre;            // workspace: [T][4] pre-mix weights (Sinkhorn kernel -> pre-mix kernel)
  int* err;              // device error word (bounded waits of the pre-mix ring)
};
size_t hc_partials_bytes(int T, int splits);
int hc_max_d();  // largest D of the pre-mix kernel (the pre-mix is held in registers)
// the per-token kernels: add p.splits partials and run the Sinkhorn split (a warp
// per token), then pre-mix, RMSNorm (+ act_quant)
cudaError_t launch_hc_pre_norm(const HcParams& p, int num_sms, cudaStream_t stream);
// mixing partials on the tensor cores (hc_tc.cu): fn [nmix][KD] -> parts bf16
// [3][32][KD]; x_flat [T][KD] and the parts as 128-byte-swizzled 64-wide maps
// (128-row and 32-row boxes)
int hc_mix_tc_splits(int T, int KD, int num_sms);
size_t hc_fn_parts_bytes(int KD);
cudaError_t launch_hc_split_fn(const float* fn, int nmix, int KD, void* parts, int num_sms, cudaStream_t stream);
cudaError_t launch_hc_mix_tc(const CUtensorMap& tmap_x, const CUtensorMap& tmap_f, int T, int KD, int nmix,
                             int splits, float* partial, int* err, cudaStream_t stream);
// standalone RMSNorm, one row per CTA (D % 8 == 0; q / q_scale optional: act_quant_ref of y)
cudaError_t launch_rms_norm(const void* x, const float* w, int T, int D, float eps, void* y, uint8_t* q,
                            float* q_scale, cudaStream_t stream);
cudaError_t launch_hc_post(const void* y, const void* residual, const float* post, const float* comb, int T, int D,
                           int hc, void* out, int num_sms, cudaStream_t stream);

// ---- layout (layout.cu)
struct LayoutParams {
  const int64_t* idx;     // [T][k]
  const float* weights;   // [T][k] or null (1.0)
  int T, k, E;
  int with_shared;
  const int* T_dev;          // optional: token count read on the device (<= T)
  int tt_routed, tt_shared;  // token rows per GEMM tile
  int rpad_to_tile;          // 1: every tile's rows are padded to the tile size (two-plane tiles), else to 16
  int max_tiles;
  int* counts;            // [E+1]
  int* offsets;           // [E+2]
  int* row_of;            // [T][k]
  int* row_sorted;        // [T][k] rows of each token in ascending expert id
  int* row_token;         // [R]
  float* row_weight;      // [R]
  int* row_tile;          // [R] token tile holding the row
  int* row_pos;           // [R] (rpad of that tile << 8) | position of the row in it
  int* tiles;             // [max_tiles][3]
  int* n_tiles;
  int* err;
  int* scratch;           // layout_scratch_ints(T, k, E) ints: the multi-CTA layout of
                          // batches above 1024 assignments (null: the single-CTA kernel)
  int pad_ok;             // 1: negative ids are padding slots (no row, no error)
};
size_t layout_scratch_ints(int T, int k, int E);
cudaError_t launch_layout(const LayoutParams& p, cudaStream_t stream);
cudaError_t launch_layout_assignments(const int64_t* ids, int A, int E, int64_t* sorted_ids, int64_t* perm,
                                      int32_t* offsets, int32_t* counts, cudaStream_t stream);
cudaError_t launch_emit_tiles(const int32_t* counts, int E, int block_m, int max_tiles, int32_t* expert_index,
                              int32_t* m_start, int32_t* n_tiles, int32_t* tile_rows, cudaStream_t stream);

// ---- quantisation (quant.cu)
// x bf16 [T][ldx] (first H values of each row used) -> packed activation rows:
// row_of[t][s] (s < k) and, when shared_base >= 0, row shared_base + t.
// hilo: hi/lo planes with per-32 scales; else act_quant_ref per 128.  Rows are
// stored K-tile-major, xq[H/128][planes][R_pad][128 B]; scales go straight into
// the token tile's MMA scale chunks sft [tile][H/128][128 words].
cudaError_t launch_rows_quant(const void* x, int T, const int* T_dev, int H, int ldx, int k, const int* row_of,
                              int shared_base, int hilo, int R_pad, const int* row_tile, const int* row_pos,
                              uint8_t* xq, uint32_t* sft, cudaStream_t stream);
// E4M3 exchange rows (codes [H], biased scale exponents [H/128] padded to 16
// bytes, then the meta tail) -> the same packed planes and scale chunks as
// launch_rows_quant in act_quant_ref mode: row r goes to packed row row_of[r]
// (rows with row_of < 0 are skipped); with R_dev only the first *R_dev rows.
cudaError_t launch_rows_place_e4m3(const void* rows, int row_bytes, int R, const int* R_dev, int H, const int* row_of,
                                   int R_pad, const int* row_tile, const int* row_pos, uint8_t* xq, uint32_t* sft,
                                   cudaStream_t stream);
// E4M3 unit rows (MOSAIC_EP_ROW_BYTES_E4M3_UNITS) -> the same planes and scale
// chunks: unit u's codes to the packed row of each used slot (row_of[u*K + j]),
// and row_rank / row_ret [R] = slot j's return rank and position (a_rank / a_pos
// [U*K]) under that packed row; only the first *U_dev units.
cudaError_t launch_rows_place_units(const void* rows, int row_bytes, int U, const int* U_dev, int H, int K,
                                    const int* row_of, const int* a_rank, const int* a_pos, int R_pad,
                                    const int* row_tile, const int* row_pos, uint8_t* xq, uint32_t* sft,
                                    int* row_rank, int* row_ret, cudaStream_t stream);
cudaError_t launch_act_quant(const void* x, int M, int K, uint8_t* q, float* scale, cudaStream_t stream);
cudaError_t launch_pack_mxfp4(const float* w, int N, int K, uint8_t* packed, uint8_t* scale, cudaStream_t stream);
// halves = 2 interleaves the two row halves of each matrix (gate rows, up rows)
// per (row block, K-tile): tile order [mat][row block][K-tile][half].
cudaError_t launch_repack_weights(const uint8_t* packed, int n_mats, int rows, int K, int halves, uint8_t* tiled,
                                  cudaStream_t stream);
cudaError_t launch_prepack_scales(const uint8_t* scale, int n_mats, int rows, int K, int halves, uint8_t* chunks,
                                  cudaStream_t stream);

// ---- expert parallelism (ep.cu)
// Send rows of one rank, in the layout's expert-sorted row order: row r holds
// x[row_token[r]] (H bf16) then a 16-byte tail {local expert id, route weight
// bits, source token, destination rank} (int32 each).  dest_counts[d] = rows
// for rank d = experts [d*E_local, (d+1)*E_local).
cudaError_t launch_ep_pack(const void* x, int H, int A, int E, int E_local, int world, const int* offsets,
                           const int* row_token, const float* row_weight, void* send, int* dest_counts,
                           cudaStream_t stream);
// Per-row expert ids / weights with an element stride (ids null: every row
// uses default_id; weights null: 1.0) -> int64 idx [R], fp32 w [R]; ids outside
// [0, E) are recorded as MOSAIC_ERR_RANGE and replaced by 0 with weight 0.
// rows_dev (optional): only the first *rows_dev rows are read.
cudaError_t launch_rows_meta(const int32_t* ids, const float* weights, int stride, int R, const int* rows_dev, int E,
                             int default_id, int64_t* idx, float* w, int* err, cudaStream_t stream);

// Exchange region of one rank (peer-memory EP): this header, then the receive
// rows, then the return partials.
struct EpRegionHeader {
  int err;                   // device error word (first: mosaic_read_error reads it)
  int err_pad[3];            // mosaic_read_error's reset clears 16 bytes: nothing else lives here
  uint32_t epoch;            // step counter, advanced by the count exchange
  uint32_t send_done;        // CTAs of the row copy that finished (last one signals)
  uint32_t ret_done;         // same for the partial copy
  int recv_count;            // rows received in the current step
  int pad[3];
  uint32_t count_flag[MOSAIC_EP_MAX_WORLD];  // [source]: its counts of this epoch are here
  uint32_t data_flag[MOSAIC_EP_MAX_WORLD];   // [source]: its rows of this epoch are here
  uint32_t ret_flag[MOSAIC_EP_MAX_WORLD];    // [owner]: its partials of this epoch are here
  int counts[MOSAIC_EP_MAX_WORLD][MOSAIC_EP_MAX_WORLD];  // [source][destination] rows
  // geometry of the step's received rows, written with the counts: rows from
  // source s are receive rows [recv_start[s], recv_start[s+1]) and go back to
  // s's send rows from src_pos[s]
  int recv_start[MOSAIC_EP_MAX_WORLD + 1];
  int src_pos[MOSAIC_EP_MAX_WORLD];
};
constexpr size_t kEpHeaderBytes = 1024;
static_assert(sizeof(EpRegionHeader) <= kEpHeaderBytes, "EP region header");

struct EpPeersDev {
  int world, rank, max_recv_rows, row_bytes, ret_row_bytes;
  unsigned long long wait_ns;  // budget of each wait on a peer's flag (global timer, ns)
  size_t recv_off, ret_off;  // byte offsets of the receive rows / return partials in a region
  uint8_t* regions[MOSAIC_EP_MAX_WORLD];
};
cudaError_t launch_ep_exchange_rows(const EpPeersDev& P, const void* send_rows, const int* dest_counts,
                                    int sms, cudaStream_t stream);
cudaError_t launch_ep_return_partials(const EpPeersDev& P, const void* partials, int sms, cudaStream_t stream);
// After a down GEMM that wrote the partials straight into the sources' return
// buffers: stamp every source's return flag, then wait for this rank's.
cudaError_t launch_ep_signal_return(const EpPeersDev& P, cudaStream_t stream);
// Unit rows (P.row_bytes = MOSAIC_EP_ROW_BYTES_E4M3_UNITS(H, K)): the units per
// owner (unit_token [world][T] scratch, dest_counts = units), the token
// quantise into tq, the count exchange, the unit send and the wait.
cudaError_t launch_ep_dispatch_send_units(const EpPeersDev& P, const void* x, int T, int H, int k, int E_local,
                                          int K, const int64_t* idx, const float* weights, const int* row_of,
                                          int* dest_counts, int* unit_token, uint8_t* tq, int sms,
                                          cudaStream_t stream);
// Received unit rows -> assignments idx / w / a_rank / a_pos [U_max * K] (id -1: unused slot).
cudaError_t launch_ep_units_meta(const EpPeersDev& P, int H, int K, int U_max, int64_t* idx, float* w, int* a_rank,
                                 int* a_pos, cudaStream_t stream);
// E4M3 rows without a send buffer: destination counts from the layout's
// offsets (kept in dest_counts), every token row quantised once (act_quant_ref)
// into tq [T][H + pad] (scratch, T * (H + 128) bytes is enough), the count
// exchange, then a warp per send row copies its token's E4M3 row straight into
// its owner's receive row, and the wait for every source's rows.
// P.row_bytes must be MOSAIC_EP_ROW_BYTES_E4M3(H).
cudaError_t launch_ep_dispatch_send_e4m3(const EpPeersDev& P, const void* x, int T, int H, int E, int E_local,
                                         const int* offsets, const int* row_token, const float* row_weight,
                                         int* dest_counts, uint8_t* tq, int sms, cudaStream_t stream);

// ---- combine (combine.cu)
cudaError_t launch_combine(const void* partial, int partial_f32, const int* row_sorted, int T, int k, int H,
                           int shared_base, void* y, cudaStream_t stream);

}  // namespace mosaic
