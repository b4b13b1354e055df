// C ABI of the Mosaic B200 MoE hot path (see include/mosaic_moe.h).
//
// Host side only: argument validation, workspace planning, TMA tensor-map
// encoding and kernel launches.  Nothing here allocates device memory or
// synchronises a stream (except mosaic_read_error, which exists to do so).
// cuTensorMapEncodeTiled is resolved through cudaGetDriverEntryPoint so the
// library does not link libcuda and loads on hosts without a GPU.
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "kernels.h"

using namespace mosaic;

// Token rows per bf16 (decode) tile; the hi + lo planes of a tile make MMA N = 32.
#define MOSAIC_DECODE_TILE_ROWS 16


namespace {

constexpr int kVersion = 1;

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = []() -> EncodeTiledFn {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess) return nullptr;
    if (q != cudaDriverEntryPointSuccess) return nullptr;
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  return n;
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

size_t up256(size_t v) { return (v + 255) & ~size_t(255); }

// Weights: 3-D map {128 values, 128 rows, tiles} over the tiled E2M1 codes; one
// box = two consecutive 8 KB tiles (gate + up of one K-tile, or two K-tiles of
// down), unpacked by TMA into the 16-byte-per-16-values smem layout that
// kind::mxf8f6f4 reads.
int make_weight_map(CUtensorMap* map, const uint8_t* tiled, int n_bank, int rows, int K, int box_tiles) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return MOSAIC_ERR_CUDA;
  const cuuint64_t n_tiles = static_cast<cuuint64_t>(n_bank) * (rows / 128) * (K / 128);
  cuuint64_t dims[3] = {128, 128, n_tiles};
  cuuint64_t strides[2] = {64, 8192};
  cuuint32_t box[3] = {128, 128, static_cast<cuuint32_t>(box_tiles)};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, 3, const_cast<uint8_t*>(tiled), dims, strides, box,
                   es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? MOSAIC_OK : MOSAIC_ERR_CUDA;
}

// Activations: 4-D map {128 bytes, rows, planes, K-tiles} over E4M3 rows stored
// K-tile-major ([K/128][planes][R_pad][128 B]); one box = brows rows of every
// plane for ks consecutive K-tiles.
int make_act_map(CUtensorMap* map, const uint8_t* q, int R_pad, int planes, int K, int brows, int ks) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return MOSAIC_ERR_CUDA;
  cuuint64_t dims[4] = {128, static_cast<cuuint64_t>(R_pad), static_cast<cuuint64_t>(planes),
                        static_cast<cuuint64_t>(K / 128)};
  cuuint64_t strides[3] = {128, static_cast<cuuint64_t>(R_pad) * 128, static_cast<cuuint64_t>(planes) * R_pad * 128};
  cuuint32_t box[4] = {128, static_cast<cuuint32_t>(brows), static_cast<cuuint32_t>(planes),
                       static_cast<cuuint32_t>(ks)};
  cuuint32_t es[4] = {1, 1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<uint8_t*>(q), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? MOSAIC_OK : MOSAIC_ERR_CUDA;
}

// Router logits on the tensor cores (router_tc.cu) wherever the shape allows.
// W is split into three bf16 parts once per call into the workspace, except
// for the smallest batches, whose logits kernel splits it in shared memory.
bool router_tc_parts(int T, int H, int E, int sms) {
  return router_tc_applies(H, E) && !router_tc_convert(T, H, E, sms);
}

size_t router_parts_bytes(int T, int H, int E, int sms) {
  return router_tc_parts(T, H, E, sms) ? up256(sizeof(uint16_t) * 3 * static_cast<size_t>(E) * H) : 0;
}

int make_bf16_rows_map(CUtensorMap* map, const void* base, int rows, int K, int box_rows = 128) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return MOSAIC_ERR_CUDA;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(K) * 2};
  cuuint32_t box[2] = {64, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t es[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? MOSAIC_OK : MOSAIC_ERR_CUDA;
}

// W fp32 [E][H] as a 2-D map with unswizzled 64-value x 128-row boxes.
int make_f32_rows_map(CUtensorMap* map, const float* base, int rows, int K) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return MOSAIC_ERR_CUDA;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(K) * 4};
  cuuint32_t box[2] = {64, 128};
  cuuint32_t es[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? MOSAIC_OK : MOSAIC_ERR_CUDA;
}

// Logits + top-k.  splits = router_splits(T, H, E, sms) sizes the partials;
// parts (router_parts_bytes) holds W's bf16 split when the logits kernel does
// not split W itself.
int run_router(const void* x, const float* w, const float* bias, int T, int H, int E, int top_k, int n_group,
               int topk_group, float route_scale, int norm, float* weights_out, int64_t* idx_out, float* partial,
               void* parts, int splits, int* err, cudaStream_t stream, const RouteVariant* rv) {
  const RouteVariant r = rv ? *rv : RouteVariant{};
  const int sms = sm_count();
  // small batches: one launch; err[1] (zeroed with the error word by every
  // caller) counts the CTAs that finished their logits
  if (!(r.hash && !r.tid2eid) && err && router_small_applies(T, H, E))
    return launch_router_small(x, w, bias, T, H, E, top_k, n_group, topk_group, route_scale, norm, weights_out,
                               idx_out, partial, err + 1, err, stream, rv) == cudaSuccess
               ? MOSAIC_OK
               : MOSAIC_ERR_CUDA;
  if (!(r.hash && !r.tid2eid) && sms > 0 && router_tc_applies(H, E)) {
    const bool use_parts = router_tc_parts(T, H, E, sms);
    if (use_parts && !parts) return MOSAIC_ERR_WORKSPACE;
    CUtensorMap tx, tw;
    int st = make_bf16_rows_map(&tx, x, T, H);
    if (st) return st;
    if (use_parts) {
      if (launch_router_split_w(w, E, H, parts, sms, stream) != cudaSuccess) return MOSAIC_ERR_CUDA;
      st = make_bf16_rows_map(&tw, parts, 3 * E, H);
    } else {
      st = make_f32_rows_map(&tw, w, E, H);
    }
    if (st) return st;
    if (launch_router_logits_tc(tx, tw, !use_parts, T, H, E, splits, partial, err, stream) != cudaSuccess)
      return MOSAIC_ERR_CUDA;
    PdlScope pdl(true);  // the top-k follows the logits kernel in the stream
    return launch_router_topk(partial, splits, bias, T, E, top_k, n_group, topk_group, route_scale, norm, weights_out,
                              idx_out, err, stream, rv) == cudaSuccess
               ? MOSAIC_OK
               : MOSAIC_ERR_CUDA;
  }
  return launch_router(x, w, bias, T, H, E, top_k, n_group, topk_group, route_scale, norm, weights_out, idx_out,
                       partial, splits, err, stream, rv) == cudaSuccess
             ? MOSAIC_OK
             : MOSAIC_ERR_CUDA;
}

struct WsPlan {
  int R, R_pad, planes, max_tiles, splits, tt, n_bank, partial_f32, max_n, nbuf, parities;
  size_t err, router_part, router_parts, counts, offsets, row_of, row_sorted, row_token, row_weight, row_tile, row_pos, tiles,
      n_tiles;
  size_t xq, x_sft, zq, z_sft, partial, row_idx, row_w, lay_scratch, total;
};

int check_dims(const mosaic_moe_dims* d) {
  if (!d) return MOSAIC_ERR_SHAPE;
  if (d->tokens < 1 || d->tokens > (1 << 20)) return MOSAIC_ERR_SHAPE;
  // H: whole pairs of 128-row down blocks; I: whole 128-row gate/up blocks
  if (d->hidden < 256 || d->hidden % 256 || d->inter < 128 || d->inter % 128) return MOSAIC_ERR_SHAPE;
  if (d->n_experts < 1 || d->n_experts > 256) return MOSAIC_ERR_UNSUPPORTED;
  if (d->top_k < 1 || d->top_k > 8 || d->top_k > d->n_experts) return MOSAIC_ERR_SHAPE;
  if (d->n_group < 1 || d->n_group > 32 || d->n_experts % d->n_group) return MOSAIC_ERR_SHAPE;
  if (d->topk_group < 1 || d->topk_group > d->n_group) return MOSAIC_ERR_SHAPE;
  if (d->topk_group * (d->n_experts / d->n_group) < d->top_k) return MOSAIC_ERR_SHAPE;
  if (d->act_mode != MOSAIC_ACT_BF16 && d->act_mode != MOSAIC_ACT_FP8) return MOSAIC_ERR_DTYPE;
  if (!(d->swiglu_limit >= 0.f)) return MOSAIC_ERR_RANGE;
  return MOSAIC_OK;
}

// rows_mode: the per-row expert pass (mosaic_moe_expert_rows) — no router
// partials and no partial buffer (the caller owns the output), plus the
// per-row expert ids / weights it unpacks.
WsPlan plan_ws(const mosaic_moe_dims* d, bool rows_mode = false) {
  WsPlan w{};
  const int T = d->tokens, H = d->hidden, I = d->inter, E = d->n_experts, k = d->top_k;
  const bool hilo = d->act_mode == MOSAIC_ACT_BF16;
  (void)I;
  w.n_bank = E + (d->has_shared ? 1 : 0);
  w.R = T * k + (d->has_shared ? T : 0);
  w.R_pad = (w.R + 15) & ~15;
  w.planes = hilo ? 2 : 1;
  // Token rows per tile.  bf16 (decode) tiles carry hi + lo planes: MMA N = 2 * rows.
  // When the batch averages 16 or more rows per expert (e.g. the receive side
  // of expert parallelism), 32-row tiles stop a second tile from streaming the
  // same expert's weights again; they use one TMEM accumulator buffer
  // (3 parities x 2 x 64 columns + 48 scale columns) instead of two.
  // E4M3 (prefill) tiles hold 112 rows so that two accumulator buffers fit TMEM
  // (2 x 2 x 112 columns + 32 scale columns <= 512): the epilogue of one work
  // item then overlaps the MMAs of the next instead of stalling them.
  const bool wide = hilo && w.R >= 16 * w.n_bank;
  w.tt = hilo ? (wide ? 2 * MOSAIC_DECODE_TILE_ROWS : MOSAIC_DECODE_TILE_ROWS) : 112;
  w.max_n = hilo ? 2 * w.tt : w.tt;
  // sum over experts of ceil(count / tt) <= A / tt + (experts with a partial tile)
  w.max_tiles = (T * k) / w.tt + w.n_bank + T / w.tt + 2;
  // Two TMEM accumulator buffers (one for wide decode tiles); decode tiles
  // (small N, issue-bound) use three stage parities (six MMA issuers),
  // prefill tiles one.
  w.nbuf = wide ? 1 : 2;
  w.parities = hilo ? 3 : 1;
  const int sms = sm_count();
  w.splits = router_splits(T, H, E, sms > 0 ? sms : 148);
  w.partial_f32 = hilo ? 1 : 0;
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o = up256(o + bytes);
    return at;
  };
  w.err = take(16);
  w.router_part = take(rows_mode ? 0 : sizeof(float) * static_cast<size_t>(w.splits) * T * E);
  w.router_parts = take(rows_mode ? 0 : router_parts_bytes(T, H, E, sms > 0 ? sms : 148));
  w.counts = take(sizeof(int) * (E + 1));
  w.offsets = take(sizeof(int) * (E + 2));
  w.row_of = take(sizeof(int) * static_cast<size_t>(T) * k);
  w.row_sorted = take(sizeof(int) * static_cast<size_t>(T) * k);
  w.row_token = take(sizeof(int) * static_cast<size_t>(w.R));
  w.row_weight = take(sizeof(float) * static_cast<size_t>(w.R));
  w.row_tile = take(sizeof(int) * static_cast<size_t>(w.R));
  w.row_pos = take(sizeof(int) * static_cast<size_t>(w.R));
  w.tiles = take(sizeof(int) * 3 * static_cast<size_t>(w.max_tiles));
  w.n_tiles = take(sizeof(int) * 4);
  w.xq = take(static_cast<size_t>(w.planes) * w.R_pad * H);
  w.x_sft = take(static_cast<size_t>(w.max_tiles) * (H / 128) * 512);
  w.zq = take(static_cast<size_t>(w.planes) * w.R_pad * I);
  w.z_sft = take(static_cast<size_t>(w.max_tiles) * (I / 128) * 512);
  w.partial = take(rows_mode ? 0 : static_cast<size_t>(w.R) * H * (w.partial_f32 ? 4 : 2));
  w.row_idx = take(rows_mode ? sizeof(int64_t) * static_cast<size_t>(T) : 0);
  w.row_w = take(rows_mode ? sizeof(float) * static_cast<size_t>(T) : 0);
  w.lay_scratch = take(sizeof(int) * layout_scratch_ints(T, k, E));
  w.total = o;
  return w;
}

int check_bank(const mosaic_expert_bank* b) {
  if (!b || !b->gu_tiled || !b->gu_sf || !b->dn_tiled || !b->dn_sf) return MOSAIC_ERR_SHAPE;
  if (!aligned(b->gu_tiled, 32) || !aligned(b->dn_tiled, 32)) return MOSAIC_ERR_ALIGN;
  if (!aligned(b->gu_sf, 16) || !aligned(b->dn_sf, 16)) return MOSAIC_ERR_ALIGN;
  return MOSAIC_OK;
}

// Layout -> quantise -> gate/up -> down -> combine, with routing in
// (idx, weights) already on the device.
// ev (optional) = 7 events: before router, after router, layout, quantise,
// gate/up, down, combine; slots 0-1 are recorded by the caller of run_experts.
// Launch groups of the expert pass: layout + quantise + gate/up, and down +
// combine.  The fused entry points run both; mosaic_expert_gemm_gu and
// mosaic_expert_gemm_down run one each over a shared workspace.
constexpr int kStageGateUp = 1;
constexpr int kStageDown = 2;

inline bool rec(void* const* ev, int i, cudaStream_t s) {
  return !ev || !ev[i] || cudaEventRecord(static_cast<cudaEvent_t>(ev[i]), s) == cudaSuccess;
}

void fill_layout(LayoutParams& lp, const WsPlan& w, uint8_t* ws) {
  lp.tt_routed = w.tt;
  lp.tt_shared = w.tt;
  lp.rpad_to_tile = w.planes == 2 ? 1 : 0;
  lp.max_tiles = w.max_tiles;
  lp.counts = reinterpret_cast<int*>(ws + w.counts);
  lp.offsets = reinterpret_cast<int*>(ws + w.offsets);
  lp.row_of = reinterpret_cast<int*>(ws + w.row_of);
  lp.row_sorted = reinterpret_cast<int*>(ws + w.row_sorted);
  lp.row_token = reinterpret_cast<int*>(ws + w.row_token);
  lp.row_weight = reinterpret_cast<float*>(ws + w.row_weight);
  lp.row_tile = reinterpret_cast<int*>(ws + w.row_tile);
  lp.row_pos = reinterpret_cast<int*>(ws + w.row_pos);
  lp.tiles = reinterpret_cast<int*>(ws + w.tiles);
  lp.n_tiles = reinterpret_cast<int*>(ws + w.n_tiles);
  lp.err = reinterpret_cast<int*>(ws + w.err);
  lp.scratch = layout_scratch_ints(lp.T, lp.k, lp.E) ? reinterpret_cast<int*>(ws + w.lay_scratch) : nullptr;
}

// Gate/up (+ SwiGLU, route weight, re-quantisation) then down over the packed
// rows the layout and rows_quant left in the workspace.  Down partials go to
// partial_out, row r at out_row[r] (out_row null: row r).  stages selects the
// launches: a down-only pass reads the z rows and tile list an earlier
// gate/up-only pass left in the same workspace.
int run_gemms(const mosaic_moe_dims* d, const WsPlan& w, uint8_t* ws, const LayoutParams& lp,
              const mosaic_expert_bank* bank, int shared_expert, const int* out_row, void* partial_out,
              cudaStream_t stream, void* const* ev, const EpPeersDev* ep = nullptr,
              const int* expert_slot = nullptr, int bank_slots = 0, const int* ep_row_rank = nullptr,
              const int* ep_row_pos = nullptr, int stages = kStageGateUp | kStageDown) {
  const int n_map = expert_slot ? bank_slots : w.n_bank;  // bank entries the weight maps cover
  const int H = d->hidden, I = d->inter;
  const bool hilo = d->act_mode == MOSAIC_ACT_BF16;
  const int sms = sm_count();
  if (sms <= 0) return MOSAIC_ERR_CUDA;
  CUtensorMap tw, tx;
  GemmParams gp{};
  gp.hilo = hilo ? 1 : 0;
  gp.fp8 = hilo ? 0 : 1;
  gp.I = I;
  gp.H = H;
  gp.R = w.R;
  gp.R_pad = w.R_pad;
  gp.shared_expert = shared_expert;
  gp.tiles = lp.tiles;
  gp.n_tiles = lp.n_tiles;
  gp.max_tiles = w.max_tiles;
  gp.row_weight = lp.row_weight;
  gp.max_n = w.max_n;
  gp.brows = w.tt;
  gp.nbuf = w.nbuf;
  gp.swiglu_limit = d->swiglu_limit;
  gp.expert_slot = expert_slot;
  gp.bank_slots = n_map;
  // the copier pays off for double-buffered two-plane (decode) tiles; with one
  // buffer (wide decode tiles) or E4M3 tiles its extra hop per stage costs more
  // than it saves
  gp.sf_copier = (w.nbuf == 2 && hilo) ? 1 : 0;
  gp.err = lp.err;

  // gate/up
  int st = make_weight_map(&tw, bank->gu_tiled, n_map, 2 * I, H, 2);
  if (st) return st;
  st = make_act_map(&tx, ws + w.xq, w.R_pad, w.planes, H, w.tt, 1);
  if (st) return st;
  gp.mode = 0;
  gp.parities = w.parities;
  gp.K = H;
  gp.n_blocks = I / 128;
  gp.x_sft = ws + w.x_sft;
  gp.w_sf = bank->gu_sf;
  gp.zq = ws + w.zq;
  gp.z_sft = reinterpret_cast<uint32_t*>(ws + w.z_sft);
  if (stages & kStageGateUp) {
    if (launch_moe_gemm(tw, tx, gp, sms, stream) != cudaSuccess) return MOSAIC_ERR_CUDA;
    if (!rec(ev, 4, stream)) return MOSAIC_ERR_CUDA;
  }
  if (!(stages & kStageDown)) return MOSAIC_OK;

  // down: pairs of hidden blocks (nb, nb + H/256), adjacent in the bank
  st = make_weight_map(&tw, bank->dn_tiled, n_map, H, I, 2);
  if (st) return st;
  st = make_act_map(&tx, gp.zq, w.R_pad, w.planes, I, w.tt, 1);
  if (st) return st;
  gp.mode = 1;
  gp.parities = w.parities;
  gp.K = I;
  gp.n_blocks = H / 256;
  gp.x_sft = ws + w.z_sft;
  gp.w_sf = bank->dn_sf;
  gp.out = partial_out;
  gp.out_f32 = w.partial_f32;
  gp.out_row = out_row;
  if (ep) {  // partials go straight into the source ranks' return buffers
    const EpRegionHeader* own = reinterpret_cast<const EpRegionHeader*>(ep->regions[ep->rank]);
    gp.ep_world = ep->world;
    gp.ep_recv_start = own->recv_start;
    gp.ep_src_pos = own->src_pos;
    gp.ep_row_rank = ep_row_rank;
    gp.ep_row_pos = ep_row_pos;
    gp.ep_ret_off = ep->ret_off;
    for (int r = 0; r < ep->world; ++r) gp.ep_regions[r] = ep->regions[r];
  }
  if (launch_moe_gemm(tw, tx, gp, sms, stream) != cudaSuccess) return MOSAIC_ERR_CUDA;
  if (!rec(ev, 5, stream)) return MOSAIC_ERR_CUDA;
  return MOSAIC_OK;
}

// after_kernel: the layout follows a kernel of the layer (the router's top-k)
// in the stream, so it may launch programmatically too.
int run_experts(const mosaic_moe_dims* d, const WsPlan& w, uint8_t* ws, const void* x, const int64_t* idx,
                const float* weights, const mosaic_expert_bank* bank, void* y, cudaStream_t stream,
                void* const* ev = nullptr, const int* expert_slot = nullptr, int bank_slots = 0,
                bool after_kernel = false, int stages = kStageGateUp | kStageDown) {
  const int T = d->tokens, H = d->hidden, E = d->n_experts, k = d->top_k;
  const bool hilo = d->act_mode == MOSAIC_ACT_BF16;
  const int shared_base = d->has_shared ? T * k : -1;
  const bool gate_up = (stages & kStageGateUp) != 0;

  LayoutParams lp{};
  lp.idx = idx;
  lp.weights = weights;
  lp.T = T;
  lp.k = k;
  lp.E = E;
  lp.with_shared = d->has_shared ? 1 : 0;
  fill_layout(lp, w, ws);
  // layout -> quantise -> gate/up -> down -> combine: each kernel follows the
  // previous one in the stream, so they launch programmatically (the layout
  // only when the router's top-k precedes it); with stage events in between,
  // none does, and neither does a down-only pass, whose first kernel follows
  // whatever the caller queued
  if (gate_up) {
    PdlScope pdl_layout(ev == nullptr && after_kernel);
    if (launch_layout(lp, stream) != cudaSuccess) return MOSAIC_ERR_CUDA;
  }
  PdlScope pdl(ev == nullptr && gate_up);
  if (gate_up) {
    if (!rec(ev, 2, stream)) return MOSAIC_ERR_CUDA;
    if (launch_rows_quant(x, T, nullptr, H, H, k, lp.row_of, shared_base, hilo ? 1 : 0, w.R_pad, lp.row_tile,
                          lp.row_pos, ws + w.xq, reinterpret_cast<uint32_t*>(ws + w.x_sft), stream) != cudaSuccess)
      return MOSAIC_ERR_CUDA;
    if (!rec(ev, 3, stream)) return MOSAIC_ERR_CUDA;
  }

  const int st = run_gemms(d, w, ws, lp, bank, d->has_shared ? E : -1, nullptr, ws + w.partial, stream, ev, nullptr,
                           expert_slot, bank_slots, nullptr, nullptr, stages);
  if (st) return st;
  if (!(stages & kStageDown)) return MOSAIC_OK;

  if (launch_combine(ws + w.partial, w.partial_f32, lp.row_sorted, T, k, H, shared_base, y, stream) != cudaSuccess)
    return MOSAIC_ERR_CUDA;
  if (!rec(ev, 6, stream)) return MOSAIC_ERR_CUDA;
  return MOSAIC_OK;
}

// Dims of the per-row expert pass: every row is one assignment (k = 1) to one
// of the bank's experts, the shared one included as an ordinary id; no router.
// The per-row pass accepts up to 256 routed experts plus the shared one.
int check_rows_dims(const mosaic_moe_dims* r) {
  if (r->tokens < 1 || r->tokens > (1 << 20)) return MOSAIC_ERR_SHAPE;
  if (r->hidden < 256 || r->hidden % 256 || r->inter < 128 || r->inter % 128) return MOSAIC_ERR_SHAPE;
  if (r->n_experts < 1 || r->n_experts > 257) return MOSAIC_ERR_UNSUPPORTED;
  if (r->act_mode != MOSAIC_ACT_BF16 && r->act_mode != MOSAIC_ACT_FP8) return MOSAIC_ERR_DTYPE;
  if (!(r->swiglu_limit >= 0.f)) return MOSAIC_ERR_RANGE;
  return MOSAIC_OK;
}

mosaic_moe_dims rows_dims(const mosaic_moe_dims* d, int rows) {
  mosaic_moe_dims r = *d;
  r.tokens = rows;
  r.n_experts = d->n_experts + (d->has_shared ? 1 : 0);
  r.top_k = 1;
  r.n_group = 1;
  r.topk_group = 1;
  r.has_shared = 0;
  return r;
}

}  // namespace

// Scratch of mosaic_router_noalloc: the error word at byte 0, the split-K
// logit partials from byte 256 (the same layout as a mosaic_router workspace).
// Zero-initialised when the module loads; shared by every call on a device.
static __device__ __align__(256) uint8_t g_router_scratch[MOSAIC_ROUTER_NOALLOC_SCRATCH_BYTES];

namespace {

// Per-row expert pass; rows_dev (optional) holds the row count on the device
// (at most `rows`, which sizes the workspace and the launches).
int expert_rows_impl(const mosaic_moe_dims* dims, int32_t rows, const int32_t* rows_dev, const void* x_rows,
                     int32_t ldx, const int32_t* ids, const float* weights, int32_t meta_stride, int32_t default_id,
                     const mosaic_expert_bank* bank, void* partials, void* workspace, size_t workspace_bytes,
                     mosaic_stream_t stream, const EpPeersDev* ep = nullptr, int e4m3_row_bytes = 0) {
  if (!dims) return MOSAIC_ERR_SHAPE;
  if (rows < 0) return MOSAIC_ERR_SHAPE;
  if (e4m3_row_bytes && dims->act_mode != MOSAIC_ACT_FP8) return MOSAIC_ERR_SHAPE;
  if (rows == 0) return MOSAIC_OK;
  if (dims->n_experts > 256) return MOSAIC_ERR_UNSUPPORTED;
  const mosaic_moe_dims r = rows_dims(dims, rows);
  int st = check_rows_dims(&r);
  if (st) return st;
  if (!x_rows || (!partials && !ep) || !workspace) return MOSAIC_ERR_SHAPE;
  if (ldx < dims->hidden || ldx % 8 || ((ids || weights) && meta_stride < 1)) return MOSAIC_ERR_SHAPE;
  if (!ids && (default_id < 0 || default_id >= r.n_experts)) return MOSAIC_ERR_RANGE;
  st = check_bank(bank);
  if (st) return st;
  if (!aligned(x_rows, 16) || !aligned(partials, 16) || !aligned(workspace, 256)) return MOSAIC_ERR_ALIGN;
  if ((ids && !aligned(ids, 4)) || (weights && !aligned(weights, 4)) || (rows_dev && !aligned(rows_dev, 4)))
    return MOSAIC_ERR_ALIGN;
  const WsPlan w = plan_ws(&r, true);
  if (workspace_bytes < w.total) return MOSAIC_ERR_WORKSPACE;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  if (cudaMemsetAsync(ws + w.err, 0, 16, s) != cudaSuccess) return MOSAIC_ERR_CUDA;
  int64_t* idx = reinterpret_cast<int64_t*>(ws + w.row_idx);
  float* wt = reinterpret_cast<float*>(ws + w.row_w);
  if (launch_rows_meta(ids, weights, meta_stride, rows, rows_dev, r.n_experts, default_id, idx, wt,
                       reinterpret_cast<int*>(ws + w.err), s) != cudaSuccess)
    return MOSAIC_ERR_CUDA;
  LayoutParams lp{};
  lp.idx = idx;
  lp.weights = wt;
  lp.T = rows;
  lp.k = 1;
  lp.E = r.n_experts;
  lp.with_shared = 0;
  fill_layout(lp, w, ws);
  lp.T_dev = rows_dev;
  lp.row_sorted = nullptr;
  if (launch_layout(lp, s) != cudaSuccess) return MOSAIC_ERR_CUDA;
  const bool hilo = r.act_mode == MOSAIC_ACT_BF16;
  if (e4m3_row_bytes) {  // rows already quantised by the sender: into the operand planes as they are
    if (launch_rows_place_e4m3(x_rows, e4m3_row_bytes, rows, rows_dev, r.hidden, lp.row_of, w.R_pad, lp.row_tile,
                               lp.row_pos, ws + w.xq, reinterpret_cast<uint32_t*>(ws + w.x_sft), s) != cudaSuccess)
      return MOSAIC_ERR_CUDA;
  } else if (launch_rows_quant(x_rows, rows, rows_dev, r.hidden, ldx, 1, lp.row_of, -1, hilo ? 1 : 0, w.R_pad,
                               lp.row_tile, lp.row_pos, ws + w.xq, reinterpret_cast<uint32_t*>(ws + w.x_sft),
                               s) != cudaSuccess) {
    return MOSAIC_ERR_CUDA;
  }
  // with k = 1 the packed row of input row t is sorted row row_of[t], and
  // row_token[sorted row] = t: partials land in input row order
  return run_gemms(&r, w, ws, lp, bank, dims->has_shared ? dims->n_experts : -1, lp.row_token, partials, s,
                   nullptr, ep);
}

// Argument checks shared by mosaic_router and mosaic_router_noalloc.
int router_args_ok(const void* x, const float* weight, int32_t T, int32_t H, int32_t E, int32_t top_k,
                   int32_t n_group, int32_t topk_group, const float* weights_out, const int64_t* idx_out) {
  if (!x || !weight || !weights_out || !idx_out) return MOSAIC_ERR_SHAPE;
  if (T < 1 || H < 32 || H % 32 || E < 1 || E > 256 || top_k < 1 || top_k > 8 || top_k > E) return MOSAIC_ERR_SHAPE;
  if (n_group < 1 || n_group > 32 || E % n_group || topk_group < 1 || topk_group > n_group) return MOSAIC_ERR_SHAPE;
  if (topk_group * (E / n_group) < top_k) return MOSAIC_ERR_SHAPE;
  if (!aligned(x, 16) || !aligned(weight, 16)) return MOSAIC_ERR_ALIGN;
  return MOSAIC_OK;
}

// Host-side check of a router variant; fills the launch-side description.
int route_variant(const mosaic_route_ext* ext, int32_t top_k, RouteVariant* rv) {
  *rv = RouteVariant{};
  if (!ext) return MOSAIC_OK;
  if (ext->score_func < MOSAIC_SCORE_SIGMOID || ext->score_func > MOSAIC_SCORE_SOFTMAX) return MOSAIC_ERR_UNSUPPORTED;
  if ((ext->hash != 0 && ext->hash != 1) || ext->reserved != 0) return MOSAIC_ERR_SHAPE;
  rv->score_func = ext->score_func;
  rv->hash = ext->hash;
  if (!ext->hash) return MOSAIC_OK;
  if (ext->token_ids && !aligned(ext->token_ids, 8)) return MOSAIC_ERR_ALIGN;
  rv->token_ids = ext->token_ids;
  if (ext->tid2eid) {
    if (ext->table_rows < 1) return MOSAIC_ERR_SHAPE;
    if (!aligned(ext->tid2eid, 4)) return MOSAIC_ERR_ALIGN;
    rv->tid2eid = ext->tid2eid;
    rv->table_rows = ext->table_rows;
    return MOSAIC_OK;
  }
  if (ext->layer_idx < 0 || top_k != 1) return MOSAIC_ERR_SHAPE;
  rv->salt = static_cast<int32_t>((static_cast<int64_t>(ext->layer_idx) * 2654435761LL) % 2147483648LL);
  return MOSAIC_OK;
}

// True when the variant needs no logits (table-less hash routing).
bool salted_hash(const RouteVariant& rv) { return rv.hash && !rv.tid2eid; }

constexpr int kMaxDevices = 64;

// Device address of g_router_scratch on device dev.  Outside stream capture it
// is looked up again on every call (so a reloaded module after a device reset
// is followed); under capture the address cached by the last uncaptured call
// is used, because the lookup may load the module, which capture forbids.
int router_scratch(int dev, cudaStream_t stream, uint8_t** out) {
  static std::mutex mu;
  static uint8_t* addr[kMaxDevices] = {};
  if (dev < 0 || dev >= kMaxDevices) return MOSAIC_ERR_UNSUPPORTED;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  const bool capturing = cudaStreamIsCapturing(stream, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone;
  std::lock_guard<std::mutex> lock(mu);
  if (!capturing || !addr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_router_scratch) != cudaSuccess || !p) return MOSAIC_ERR_CUDA;
    addr[dev] = static_cast<uint8_t*>(p);
  }
  *out = addr[dev];
  return MOSAIC_OK;
}

}  // namespace

extern "C" {

int mosaic_version(void) { return kVersion; }

const char* mosaic_status_string(int status) {
  switch (status) {
    case MOSAIC_OK: return "ok";
    case MOSAIC_ERR_SHAPE: return "shape contract violated";
    case MOSAIC_ERR_DTYPE: return "unsupported number format";
    case MOSAIC_ERR_ALIGN: return "pointer alignment contract violated";
    case MOSAIC_ERR_RANGE: return "value out of range";
    case MOSAIC_ERR_CUDA: return "CUDA error";
    case MOSAIC_ERR_TIMEOUT: return "device pipeline wait timed out";
    case MOSAIC_ERR_UNSUPPORTED: return "configuration not supported";
    case MOSAIC_ERR_WORKSPACE: return "workspace too small";
    default: return "unknown status";
  }
}

int mosaic_device_sm_count(void) { return sm_count(); }

size_t mosaic_router_workspace_bytes(int32_t T, int32_t H, int32_t E) {
  if (T < 1 || H < 1 || E < 1) return 0;
  const int sms = sm_count();
  const int splits = router_splits(T, H, E, sms > 0 ? sms : 148);
  return up256(16) + up256(sizeof(float) * static_cast<size_t>(splits) * T * E) +
         router_parts_bytes(T, H, E, sms > 0 ? sms : 148);
}

int mosaic_router(const void* x, const float* weight, const float* bias, int32_t T, int32_t H, int32_t E,
                  int32_t top_k, int32_t n_group, int32_t topk_group, float route_scale, int32_t norm_topk_prob,
                  float* weights_out, int64_t* idx_out, void* workspace, size_t workspace_bytes,
                  mosaic_stream_t stream) {
  if (!workspace) return MOSAIC_ERR_SHAPE;
  const int st = router_args_ok(x, weight, T, H, E, top_k, n_group, topk_group, weights_out, idx_out);
  if (st != MOSAIC_OK) return st;
  if (!aligned(workspace, 256)) return MOSAIC_ERR_ALIGN;
  if (workspace_bytes < mosaic_router_workspace_bytes(T, H, E)) return MOSAIC_ERR_WORKSPACE;
  const int sms = sm_count();
  if (sms <= 0) return MOSAIC_ERR_CUDA;
  const int splits = router_splits(T, H, E, sms);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  if (cudaMemsetAsync(ws, 0, 16, reinterpret_cast<cudaStream_t>(stream)) != cudaSuccess) return MOSAIC_ERR_CUDA;
  const size_t part_bytes = up256(sizeof(float) * static_cast<size_t>(splits) * T * E);
  return run_router(x, weight, bias, T, H, E, top_k, n_group, topk_group, route_scale, norm_topk_prob, weights_out,
                    idx_out, reinterpret_cast<float*>(ws + up256(16)), ws + up256(16) + part_bytes, splits,
                    reinterpret_cast<int*>(ws), reinterpret_cast<cudaStream_t>(stream), nullptr);
}

int mosaic_router_ext(const mosaic_route_ext* ext, const void* x, const float* weight, const float* bias, int32_t T,
                      int32_t H, int32_t E, int32_t top_k, int32_t n_group, int32_t topk_group, float route_scale,
                      int32_t norm_topk_prob, float* weights_out, int64_t* idx_out, void* workspace,
                      size_t workspace_bytes, mosaic_stream_t stream) {
  RouteVariant rv;
  int st = route_variant(ext, top_k, &rv);
  if (st != MOSAIC_OK) return st;
  if (salted_hash(rv)) {  // no logits: x and weight are not read
    if (!weights_out || !idx_out) return MOSAIC_ERR_SHAPE;
    if (T < 1 || E < 1 || E > 256) return MOSAIC_ERR_SHAPE;
    cudaError_t e = launch_router(nullptr, nullptr, nullptr, T, H, E, top_k, 1, 1, route_scale, norm_topk_prob,
                                  weights_out, idx_out, nullptr, 1, nullptr, reinterpret_cast<cudaStream_t>(stream),
                                  &rv);
    return e == cudaSuccess ? MOSAIC_OK : MOSAIC_ERR_CUDA;
  }
  if (!workspace) return MOSAIC_ERR_SHAPE;
  st = router_args_ok(x, weight, T, H, E, top_k, n_group, topk_group, weights_out, idx_out);
  if (st != MOSAIC_OK) return st;
  if (!aligned(workspace, 256)) return MOSAIC_ERR_ALIGN;
  if (workspace_bytes < mosaic_router_workspace_bytes(T, H, E)) return MOSAIC_ERR_WORKSPACE;
  const int sms = sm_count();
  if (sms <= 0) return MOSAIC_ERR_CUDA;
  const int splits = router_splits(T, H, E, sms);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  if (cudaMemsetAsync(ws, 0, 16, reinterpret_cast<cudaStream_t>(stream)) != cudaSuccess) return MOSAIC_ERR_CUDA;
  const size_t part_bytes = up256(sizeof(float) * static_cast<size_t>(splits) * T * E);
  return run_router(x, weight, bias, T, H, E, top_k, n_group, topk_group, route_scale, norm_topk_prob, weights_out,
                    idx_out, reinterpret_cast<float*>(ws + up256(16)), ws + up256(16) + part_bytes, splits,
                    reinterpret_cast<int*>(ws), reinterpret_cast<cudaStream_t>(stream), &rv);
}

int mosaic_router_noalloc(const void* x, const float* weight, const float* bias, int32_t T, int32_t H, int32_t E,
                          int32_t top_k, int32_t n_group, int32_t topk_group, float route_scale,
                          int32_t norm_topk_prob, float* weights_out, int64_t* idx_out, mosaic_stream_t stream) {
  const int st = router_args_ok(x, weight, T, H, E, top_k, n_group, topk_group, weights_out, idx_out);
  if (st != MOSAIC_OK) return st;
  // Same split count (hence bit-identical results) as mosaic_router; inputs whose
  // partials do not fit the fixed scratch are rejected, never truncated.
  if (mosaic_router_workspace_bytes(T, H, E) > MOSAIC_ROUTER_NOALLOC_SCRATCH_BYTES) return MOSAIC_ERR_WORKSPACE;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return MOSAIC_ERR_CUDA;
  const int sms = sm_count();
  if (sms <= 0) return MOSAIC_ERR_CUDA;
  uint8_t* ws = nullptr;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int sst = router_scratch(dev, s, &ws);
  if (sst != MOSAIC_OK) return sst;
  if (cudaMemsetAsync(ws, 0, 16, s) != cudaSuccess) return MOSAIC_ERR_CUDA;  // this call's error word
  const int splits = router_splits(T, H, E, sms);
  const size_t part_bytes = up256(sizeof(float) * static_cast<size_t>(splits) * T * E);
  return run_router(x, weight, bias, T, H, E, top_k, n_group, topk_group, route_scale, norm_topk_prob, weights_out,
                    idx_out, reinterpret_cast<float*>(ws + up256(16)), ws + up256(16) + part_bytes, splits,
                    reinterpret_cast<int*>(ws), reinterpret_cast<cudaStream_t>(stream), nullptr);
}

int mosaic_layout_assignments(const int64_t* expert_ids, int32_t A, int32_t E, int64_t* sorted_ids, int64_t* perm,
                              int32_t* offsets, int32_t* counts, mosaic_stream_t stream) {
  if (!expert_ids || !sorted_ids || !perm || !offsets || !counts) return MOSAIC_ERR_SHAPE;
  if (A < 1 || A > (1 << 20) || E < 1 || E > 256) return MOSAIC_ERR_SHAPE;
  cudaError_t e = launch_layout_assignments(expert_ids, A, E, sorted_ids, perm, offsets, counts,
                                            reinterpret_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MOSAIC_OK : MOSAIC_ERR_CUDA;
}

int mosaic_emit_tiles(const int32_t* counts, int32_t E, int32_t block_m, int32_t max_tiles, int32_t* expert_index,
                      int32_t* m_start, int32_t* n_tiles, int32_t* tile_rows, mosaic_stream_t stream) {
  if (!counts || !expert_index || !m_start || !n_tiles || !tile_rows) return MOSAIC_ERR_SHAPE;
  if (E < 1 || E > 4096 || block_m < 1 || max_tiles < 0) return MOSAIC_ERR_SHAPE;
  cudaError_t e = launch_emit_tiles(counts, E, block_m, max_tiles, expert_index, m_start, n_tiles, tile_rows,
                                    reinterpret_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MOSAIC_OK : MOSAIC_ERR_CUDA;
}

int mosaic_act_quant(const void* x, int32_t M, int32_t K, uint8_t* q, float* scale, mosaic_stream_t stream) {
  if (!x || !q || !scale) return MOSAIC_ERR_SHAPE;
  if (M < 1 || K < 128 || K % 128) return MOSAIC_ERR_SHAPE;
  if (!aligned(x, 16) || !aligned(q, 8)) return MOSAIC_ERR_ALIGN;
  cudaError_t e = launch_act_quant(x, M, K, q, scale, reinterpret_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MOSAIC_OK : MOSAIC_ERR_CUDA;
}

int mosaic_pack_mxfp4(const float* w, int32_t N, int32_t K, uint8_t* packed, uint8_t* scale,
                      mosaic_stream_t stream) {
  if (!w || !packed || !scale) return MOSAIC_ERR_SHAPE;
  if (N < 1 || K < 32 || K % 32) return MOSAIC_ERR_SHAPE;
  if (!aligned(w, 16) || !aligned(packed, 16)) return MOSAIC_ERR_ALIGN;
  cudaError_t e = launch_pack_mxfp4(w, N, K, packed, scale, reinterpret_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MOSAIC_OK : MOSAIC_ERR_CUDA;
}

int mosaic_repack_weights(const uint8_t* packed, int32_t n_mats, int32_t rows, int32_t K, int32_t halves,
                          uint8_t* tiled, mosaic_stream_t stream) {
  if (!packed || !tiled) return MOSAIC_ERR_SHAPE;
  if (halves != 1 && halves != 2) return MOSAIC_ERR_SHAPE;
  if (n_mats < 1 || rows < 128 * halves || rows % (128 * halves) || K < 128 || K % 128) return MOSAIC_ERR_SHAPE;
  if (!aligned(packed, 16) || !aligned(tiled, 16)) return MOSAIC_ERR_ALIGN;
  cudaError_t e =
      launch_repack_weights(packed, n_mats, rows, K, halves, tiled, reinterpret_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MOSAIC_OK : MOSAIC_ERR_CUDA;
}

int mosaic_prepack_scales(const uint8_t* scale, int32_t n_mats, int32_t rows, int32_t K, int32_t halves,
                          uint8_t* sf_chunks, mosaic_stream_t stream) {
  if (!scale || !sf_chunks) return MOSAIC_ERR_SHAPE;
  if (halves != 1 && halves != 2) return MOSAIC_ERR_SHAPE;
  if (n_mats < 1 || rows < 128 * halves || rows % (128 * halves) || K < 128 || K % 128) return MOSAIC_ERR_SHAPE;
  cudaError_t e =
      launch_prepack_scales(scale, n_mats, rows, K, halves, sf_chunks, reinterpret_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MOSAIC_OK : MOSAIC_ERR_CUDA;
}

// Workspace of mosaic_hc_pre_norm: [error word][partials][fn parts].
struct HcWs {
  int splits;
  size_t partial, parts, pre, total;
};
HcWs hc_ws(int T, int D, int hc, int sms) {
  HcWs w{};
  w.splits = hc_mix_tc_splits(T, hc * D, sms);
  w.partial = 256;
  w.parts = w.partial + up256(hc_partials_bytes(T, w.splits));
  w.pre = w.parts + up256(hc_fn_parts_bytes(hc * D));
  w.total = w.pre + up256(static_cast<size_t>(T) * 4 * sizeof(float));
  return w;
}

size_t mosaic_hc_pre_norm_workspace_bytes(int32_t T, int32_t D, int32_t hc) {
  if (T < 1 || D < 128 || D % 128 || hc < 1 || hc > 4) return 0;
  const int sms = sm_count();
  return hc_ws(T, D, hc, sms > 0 ? sms : 148).total;
}

int mosaic_hc_pre_norm(const void* x, const float* fn, const float* base, const float* scale,
                       const float* norm_weight, int32_t T, int32_t D, int32_t hc, int32_t sinkhorn_iters,
                       float hc_eps, float norm_eps, void* y, float* post, float* comb, uint8_t* q, float* q_scale,
                       void* workspace, size_t workspace_bytes, mosaic_stream_t stream) {
  if (!x || !fn || !base || !scale || !y || !post || !comb || !workspace) return MOSAIC_ERR_SHAPE;
  if ((q == nullptr) != (q_scale == nullptr)) return MOSAIC_ERR_SHAPE;
  if (T < 1 || D < 128 || D % 128 || hc < 1 || hc > 4 || sinkhorn_iters < 1) return MOSAIC_ERR_SHAPE;
  if (!aligned(x, 16) || !aligned(fn, 16) || (norm_weight && !aligned(norm_weight, 16)) || !aligned(y, 16) ||
      (q && !aligned(q, 16)))
    return MOSAIC_ERR_ALIGN;
  if (!aligned(workspace, 256)) return MOSAIC_ERR_ALIGN;
  const int sms = sm_count();
  if (sms <= 0) return MOSAIC_ERR_CUDA;
  if (D > hc_max_d()) return MOSAIC_ERR_UNSUPPORTED;
  const HcWs w = hc_ws(T, D, hc, sms);
  if (workspace_bytes < w.total) return MOSAIC_ERR_WORKSPACE;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int KD = hc * D, nmix = (2 + hc) * hc;
  CUtensorMap tx, tf;
  int st = make_bf16_rows_map(&tx, x, T, KD);
  if (st) return st;
  st = make_bf16_rows_map(&tf, ws + w.parts, 3 * 32, KD, 3 * 32);  // one box: the three parts of a K slice
  if (st) return st;
  if (cudaMemsetAsync(ws, 0, 16, s) != cudaSuccess) return MOSAIC_ERR_CUDA;
  if (launch_hc_split_fn(fn, nmix, KD, ws + w.parts, sms, s) != cudaSuccess) return MOSAIC_ERR_CUDA;
  if (launch_hc_mix_tc(tx, tf, T, KD, nmix, w.splits, reinterpret_cast<float*>(ws + w.partial),
                       reinterpret_cast<int*>(ws), s) != cudaSuccess)
    return MOSAIC_ERR_CUDA;
  HcParams p{};
  p.partial = reinterpret_cast<float*>(ws + w.partial);
  p.splits = w.splits;
  p.x = x;
  p.fn = fn;
  p.base = base;
  p.scale = scale;
  p.norm_w = norm_weight;
  p.T = T;
  p.D = D;
  p.hc = hc;
  p.iters = sinkhorn_iters;
  p.hc_eps = hc_eps;
  p.norm_eps = norm_eps;
  p.y = y;
  p.post = post;
  p.comb = comb;
  p.q = q;
  p.q_scale = q_scale;
  p.pre = reinterpret_cast<float*>(ws + w.pre);
  p.err = reinterpret_cast<int*>(ws);
  cudaError_t e = launch_hc_pre_norm(p, sms, s);
  return e == cudaSuccess ? MOSAIC_OK : MOSAIC_ERR_CUDA;
}

int mosaic_hc_post(const void* y, const void* residual, const float* post, const float* comb, int32_t T, int32_t D,
                   int32_t hc, void* out, mosaic_stream_t stream) {
  if (!y || !residual || !post || !comb || !out) return MOSAIC_ERR_SHAPE;
  if (T < 1 || D < 8 || D % 8 || hc < 1 || hc > 4) return MOSAIC_ERR_SHAPE;
  if (!aligned(y, 16) || !aligned(residual, 16) || !aligned(out, 16)) return MOSAIC_ERR_ALIGN;
  const int sms = sm_count();
  if (sms <= 0) return MOSAIC_ERR_CUDA;
  cudaError_t e = launch_hc_post(y, residual, post, comb, T, D, hc, out, sms, reinterpret_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MOSAIC_OK : MOSAIC_ERR_CUDA;
}

int mosaic_rms_norm(const void* x, const float* weight, int32_t T, int32_t D, float eps, void* y, uint8_t* q,
                    float* q_scale, mosaic_stream_t stream) {
  if (!x || !weight || !y || ((q == nullptr) != (q_scale == nullptr))) return MOSAIC_ERR_SHAPE;
  if (T < 1 || D < 8 || D % 8 || D > MOSAIC_RMS_NORM_MAX_D) return MOSAIC_ERR_SHAPE;
  if (q && D % 128) return MOSAIC_ERR_SHAPE;
  if (!(eps >= 0.f)) return MOSAIC_ERR_RANGE;
  if (!aligned(x, 16) || !aligned(y, 16) || !aligned(weight, 16) || (q && (!aligned(q, 8) || !aligned(q_scale, 4))))
    return MOSAIC_ERR_ALIGN;
  cudaError_t e = launch_rms_norm(x, weight, T, D, eps, y, q, q_scale, reinterpret_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MOSAIC_OK : MOSAIC_ERR_CUDA;
}

size_t mosaic_moe_workspace_bytes(const mosaic_moe_dims* dims) {
  if (check_dims(dims) != MOSAIC_OK) return 0;
  return plan_ws(dims).total;
}

}  // extern "C"

namespace {

int moe_forward_impl(const mosaic_moe_dims* dims, const mosaic_route_ext* ext, const void* x,
                     const float* router_weight, const float* router_bias, const mosaic_expert_bank* bank, void* y,
                     float* weights_out, int64_t* idx_out, void* workspace, size_t workspace_bytes,
                     mosaic_stream_t stream, void* const* stage_events) {
  int st = check_dims(dims);
  if (st) return st;
  RouteVariant rv;
  st = route_variant(ext, dims->top_k, &rv);
  if (st) return st;
  const bool need_logits = !salted_hash(rv);
  if (!x || (need_logits && !router_weight) || !y || !weights_out || !idx_out || !workspace) return MOSAIC_ERR_SHAPE;
  st = check_bank(bank);
  if (st) return st;
  if (!aligned(x, 16) || !aligned(y, 16) || (need_logits && !aligned(router_weight, 16)) || !aligned(workspace, 256))
    return MOSAIC_ERR_ALIGN;
  const WsPlan w = plan_ws(dims);
  if (workspace_bytes < w.total) return MOSAIC_ERR_WORKSPACE;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  if (cudaMemsetAsync(ws + w.err, 0, 16, s) != cudaSuccess) return MOSAIC_ERR_CUDA;
  if (!rec(stage_events, 0, s)) return MOSAIC_ERR_CUDA;
  st = run_router(x, router_weight, rv.hash ? nullptr : router_bias, dims->tokens, dims->hidden, dims->n_experts,
                  dims->top_k, dims->n_group, dims->topk_group, dims->route_scale, dims->norm_topk_prob, weights_out,
                  idx_out, reinterpret_cast<float*>(ws + w.router_part), ws + w.router_parts, w.splits,
                  reinterpret_cast<int*>(ws + w.err), s, &rv);
  if (st) return st;
  if (!rec(stage_events, 1, s)) return MOSAIC_ERR_CUDA;
  return run_experts(dims, w, ws, x, idx_out, weights_out, bank, y, s, stage_events, nullptr, 0, true);
}

}  // namespace

extern "C" {

int mosaic_moe_forward_profiled(const mosaic_moe_dims* dims, const void* x, const float* router_weight,
                                const float* router_bias, const mosaic_expert_bank* bank, void* y,
                                float* weights_out, int64_t* idx_out, void* workspace, size_t workspace_bytes,
                                mosaic_stream_t stream, void* const* stage_events) {
  return moe_forward_impl(dims, nullptr, x, router_weight, router_bias, bank, y, weights_out, idx_out, workspace,
                          workspace_bytes, stream, stage_events);
}

int mosaic_moe_forward(const mosaic_moe_dims* dims, const void* x, const float* router_weight,
                       const float* router_bias, const mosaic_expert_bank* bank, void* y, float* weights_out,
                       int64_t* idx_out, void* workspace, size_t workspace_bytes, mosaic_stream_t stream) {
  return moe_forward_impl(dims, nullptr, x, router_weight, router_bias, bank, y, weights_out, idx_out, workspace,
                          workspace_bytes, stream, nullptr);
}

int mosaic_moe_forward_ext(const mosaic_moe_dims* dims, const mosaic_route_ext* ext, const void* x,
                           const float* router_weight, const float* router_bias, const mosaic_expert_bank* bank,
                           void* y, float* weights_out, int64_t* idx_out, void* workspace, size_t workspace_bytes,
                           mosaic_stream_t stream) {
  return moe_forward_impl(dims, ext, x, router_weight, router_bias, bank, y, weights_out, idx_out, workspace,
                          workspace_bytes, stream, nullptr);
}

int mosaic_moe_routed(const mosaic_moe_dims* dims, const void* x, const int64_t* expert_ids,
                      const float* expert_weights, const mosaic_expert_bank* bank, void* y, void* workspace,
                      size_t workspace_bytes, mosaic_stream_t stream) {
  int st = check_dims(dims);
  if (st) return st;
  if (!x || !expert_ids || !y || !workspace) return MOSAIC_ERR_SHAPE;
  st = check_bank(bank);
  if (st) return st;
  if (!aligned(x, 16) || !aligned(y, 16) || !aligned(workspace, 256)) return MOSAIC_ERR_ALIGN;
  const WsPlan w = plan_ws(dims);
  if (workspace_bytes < w.total) return MOSAIC_ERR_WORKSPACE;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  if (cudaMemsetAsync(ws + w.err, 0, 16, s) != cudaSuccess) return MOSAIC_ERR_CUDA;
  return run_experts(dims, w, ws, x, expert_ids, expert_weights, bank, y, s);
}

int mosaic_moe_routed_slots(const mosaic_moe_dims* dims, const void* x, const int64_t* expert_ids,
                            const float* expert_weights, const mosaic_expert_bank* bank, const int32_t* expert_slot,
                            int32_t bank_slots, void* y, void* workspace, size_t workspace_bytes,
                            mosaic_stream_t stream) {
  int st = check_dims(dims);
  if (st) return st;
  if (!x || !expert_ids || !expert_slot || !y || !workspace) return MOSAIC_ERR_SHAPE;
  if (bank_slots < 1) return MOSAIC_ERR_SHAPE;
  st = check_bank(bank);
  if (st) return st;
  if (!aligned(x, 16) || !aligned(y, 16) || !aligned(workspace, 256) || !aligned(expert_slot, 4))
    return MOSAIC_ERR_ALIGN;
  const WsPlan w = plan_ws(dims);
  if (workspace_bytes < w.total) return MOSAIC_ERR_WORKSPACE;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  if (cudaMemsetAsync(ws + w.err, 0, 16, s) != cudaSuccess) return MOSAIC_ERR_CUDA;
  return run_experts(dims, w, ws, x, expert_ids, expert_weights, bank, y, s, nullptr, expert_slot, bank_slots);
}

int mosaic_expert_gemm_gu(const mosaic_moe_dims* dims, const void* x, const int64_t* expert_ids,
                          const float* expert_weights, const mosaic_expert_bank* bank, void* workspace,
                          size_t workspace_bytes, mosaic_stream_t stream) {
  int st = check_dims(dims);
  if (st) return st;
  if (!x || !expert_ids || !workspace) return MOSAIC_ERR_SHAPE;
  st = check_bank(bank);
  if (st) return st;
  if (!aligned(x, 16) || !aligned(workspace, 256)) return MOSAIC_ERR_ALIGN;
  const WsPlan w = plan_ws(dims);
  if (workspace_bytes < w.total) return MOSAIC_ERR_WORKSPACE;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  if (cudaMemsetAsync(ws + w.err, 0, 16, s) != cudaSuccess) return MOSAIC_ERR_CUDA;
  return run_experts(dims, w, ws, x, expert_ids, expert_weights, bank, nullptr, s, nullptr, nullptr, 0, false,
                     kStageGateUp);
}

int mosaic_expert_gemm_down(const mosaic_moe_dims* dims, const mosaic_expert_bank* bank, void* y, void* workspace,
                            size_t workspace_bytes, mosaic_stream_t stream) {
  int st = check_dims(dims);
  if (st) return st;
  if (!y || !workspace) return MOSAIC_ERR_SHAPE;
  st = check_bank(bank);
  if (st) return st;
  if (!aligned(y, 16) || !aligned(workspace, 256)) return MOSAIC_ERR_ALIGN;
  const WsPlan w = plan_ws(dims);
  if (workspace_bytes < w.total) return MOSAIC_ERR_WORKSPACE;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  // the error word keeps what the gate/up call recorded
  return run_experts(dims, w, ws, nullptr, nullptr, nullptr, bank, y, s, nullptr, nullptr, 0, false, kStageDown);
}

int mosaic_ep_dispatch(const mosaic_moe_dims* dims, int32_t world, const void* x, const int64_t* idx,
                       const float* weights, void* send_rows, int32_t* dest_counts, void* workspace,
                       size_t workspace_bytes, mosaic_stream_t stream) {
  int st = check_dims(dims);
  if (st) return st;
  if (!x || !idx || !send_rows || !dest_counts || !workspace) return MOSAIC_ERR_SHAPE;
  if (world < 1 || dims->n_experts % world) return MOSAIC_ERR_SHAPE;
  if (!aligned(x, 16) || !aligned(send_rows, 16) || !aligned(workspace, 256)) return MOSAIC_ERR_ALIGN;
  const WsPlan w = plan_ws(dims);
  if (workspace_bytes < w.total) return MOSAIC_ERR_WORKSPACE;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  if (cudaMemsetAsync(ws + w.err, 0, 16, s) != cudaSuccess) return MOSAIC_ERR_CUDA;
  const int T = dims->tokens, k = dims->top_k, E = dims->n_experts;
  LayoutParams lp{};
  lp.idx = idx;
  lp.weights = weights;
  lp.T = T;
  lp.k = k;
  lp.E = E;
  lp.with_shared = 0;
  fill_layout(lp, w, ws);
  lp.row_tile = nullptr;  // no GEMM tiles on the sending side
  lp.row_pos = nullptr;
  lp.tiles = nullptr;
  if (launch_layout(lp, s) != cudaSuccess) return MOSAIC_ERR_CUDA;
  if (launch_ep_pack(x, dims->hidden, T * k, E, E / world, world, lp.offsets, lp.row_token, lp.row_weight,
                     send_rows, dest_counts, s) != cudaSuccess)
    return MOSAIC_ERR_CUDA;
  return MOSAIC_OK;
}

size_t mosaic_moe_expert_rows_workspace_bytes(const mosaic_moe_dims* dims, int32_t max_rows) {
  if (!dims || max_rows < 1) return 0;
  if (dims->n_experts > 256) return 0;
  const mosaic_moe_dims r = rows_dims(dims, max_rows);
  if (check_rows_dims(&r) != MOSAIC_OK) return 0;
  return plan_ws(&r, true).total;
}

int mosaic_moe_expert_rows(const mosaic_moe_dims* dims, int32_t rows, const void* x_rows, int32_t ldx,
                           const int32_t* ids, const float* weights, int32_t meta_stride, int32_t default_id,
                           const mosaic_expert_bank* bank, void* partials, void* workspace, size_t workspace_bytes,
                           mosaic_stream_t stream) {
  return expert_rows_impl(dims, rows, nullptr, x_rows, ldx, ids, weights, meta_stride, default_id, bank, partials,
                          workspace, workspace_bytes, stream);
}

int mosaic_moe_expert_rows_dev(const mosaic_moe_dims* dims, int32_t max_rows, const int32_t* rows_dev,
                               const void* x_rows, int32_t ldx, const int32_t* ids, const float* weights,
                               int32_t meta_stride, int32_t default_id, const mosaic_expert_bank* bank,
                               void* partials, void* workspace, size_t workspace_bytes, mosaic_stream_t stream) {
  if (!rows_dev) return MOSAIC_ERR_SHAPE;
  return expert_rows_impl(dims, max_rows, rows_dev, x_rows, ldx, ids, weights, meta_stride, default_id, bank,
                          partials, workspace, workspace_bytes, stream);
}

// ------------------------------------------------- peer-memory exchange ---

namespace {

int check_peers(const mosaic_ep_peers* p) {
  if (!p || p->world < 1 || p->world > MOSAIC_EP_MAX_WORLD || p->rank < 0 || p->rank >= p->world)
    return MOSAIC_ERR_SHAPE;
  if (p->max_recv_rows < 1 || p->max_send_rows < 1 || p->max_tokens < 1) return MOSAIC_ERR_SHAPE;
  if (p->hidden < 256 || p->hidden % 256) return MOSAIC_ERR_SHAPE;
  if (p->wait_us < 0) return MOSAIC_ERR_RANGE;
  if ((p->row_e4m3 != 0 && p->row_e4m3 != 1) || p->unit_slots < 0 || p->unit_slots > 8) return MOSAIC_ERR_SHAPE;
  if (p->unit_slots && !p->row_e4m3) return MOSAIC_ERR_SHAPE;  // unit rows are E4M3 rows
  if (p->row_e4m3 && p->partial_f32) return MOSAIC_ERR_SHAPE;  // E4M3 rows are the FP8 layer's
  if (p->row_e4m3 && p->hidden > 16384) return MOSAIC_ERR_UNSUPPORTED;
  return MOSAIC_OK;
}

size_t ep_row_bytes(const mosaic_ep_peers* p) {
  if (p->unit_slots) return MOSAIC_EP_ROW_BYTES_E4M3_UNITS(p->hidden, p->unit_slots);
  return p->row_e4m3 ? MOSAIC_EP_ROW_BYTES_E4M3(p->hidden) : MOSAIC_EP_ROW_BYTES(p->hidden);
}

// Receive-side workspace with unit rows: the per-row plan for U units of K
// slots (U * K assignments), then the assignments' ids, weights, return ranks
// and positions, and the return rank and position of every packed row.
struct UnitsWs {
  WsPlan plan;
  size_t idx, w, a_rank, a_pos, row_rank, row_ret, total;
};
UnitsWs units_ws(const mosaic_moe_dims* r) {
  UnitsWs u{};
  u.plan = plan_ws(r, true);
  const size_t A = static_cast<size_t>(r->tokens) * r->top_k;
  size_t o = u.plan.total;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o = up256(o + bytes);
    return at;
  };
  u.idx = take(sizeof(int64_t) * A);
  u.w = take(sizeof(float) * A);
  u.a_rank = take(sizeof(int) * A);
  u.a_pos = take(sizeof(int) * A);
  u.row_rank = take(sizeof(int) * static_cast<size_t>(u.plan.R));
  u.row_ret = take(sizeof(int) * static_cast<size_t>(u.plan.R));
  u.total = o;
  return u;
}

mosaic_moe_dims units_dims(const mosaic_moe_dims* d, const mosaic_ep_peers* p) {
  mosaic_moe_dims r = rows_dims(d, p->max_recv_rows);
  r.top_k = p->unit_slots;
  return r;
}

size_t ep_recv_bytes(const mosaic_ep_peers* p) { return static_cast<size_t>(p->max_recv_rows) * ep_row_bytes(p); }

int ep_ret_row_bytes(const mosaic_ep_peers* p) { return p->hidden * (p->partial_f32 ? 4 : 2); }

EpPeersDev ep_dev(const mosaic_ep_peers* p) {
  EpPeersDev d{};
  d.world = p->world;
  d.rank = p->rank;
  d.max_recv_rows = p->max_recv_rows;
  d.row_bytes = static_cast<int>(ep_row_bytes(p));
  d.ret_row_bytes = ep_ret_row_bytes(p);
  d.recv_off = kEpHeaderBytes;
  d.ret_off = up256(kEpHeaderBytes + ep_recv_bytes(p));
  d.wait_ns = p->wait_us > 0 ? static_cast<unsigned long long>(p->wait_us) * 1000ull : 2000000000ull;
  for (int r = 0; r < p->world; ++r) d.regions[r] = static_cast<uint8_t*>(p->regions[r]);
  return d;
}

int check_regions(const mosaic_ep_peers* p) {
  for (int r = 0; r < p->world; ++r)
    if (!p->regions[r] || !aligned(p->regions[r], 256)) return MOSAIC_ERR_SHAPE;
  return MOSAIC_OK;
}

}  // namespace

size_t mosaic_ep_region_bytes(const mosaic_ep_peers* peers) {
  if (check_peers(peers) != MOSAIC_OK) return 0;
  const size_t ret_rows = static_cast<size_t>(peers->max_send_rows) + peers->max_tokens;
  return up256(kEpHeaderBytes + ep_recv_bytes(peers)) + ret_rows * ep_ret_row_bytes(peers);
}

int mosaic_ep_region_alloc(size_t bytes, void** region, uint8_t* ipc_handle64) {
  if (!region || !ipc_handle64 || bytes < kEpHeaderBytes) return MOSAIC_ERR_SHAPE;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return MOSAIC_ERR_CUDA;
  // zeroed: epochs and flags start at 0 on every rank
  if (cudaMemset(p, 0, bytes) != cudaSuccess) {
    cudaFree(p);
    return MOSAIC_ERR_CUDA;
  }
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaFree(p);
    return MOSAIC_ERR_CUDA;
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  memcpy(ipc_handle64, &h, 64);
  *region = p;
  return MOSAIC_OK;
}

int mosaic_ep_region_open(const uint8_t* ipc_handle64, void** peer_region) {
  if (!ipc_handle64 || !peer_region) return MOSAIC_ERR_SHAPE;
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle64, 64);
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return MOSAIC_ERR_CUDA;
  *peer_region = p;
  return MOSAIC_OK;
}

int mosaic_ep_region_close(void* peer_region) {
  if (!peer_region) return MOSAIC_ERR_SHAPE;
  return cudaIpcCloseMemHandle(peer_region) == cudaSuccess ? MOSAIC_OK : MOSAIC_ERR_CUDA;
}

int mosaic_ep_region_free(void* region) {
  if (!region) return MOSAIC_ERR_SHAPE;
  return cudaFree(region) == cudaSuccess ? MOSAIC_OK : MOSAIC_ERR_CUDA;
}

int mosaic_ep_region_view(const mosaic_ep_peers* peers, void** recv_rows, int32_t** recv_count, void** ret_partials) {
  int st = check_peers(peers);
  if (st) return st;
  uint8_t* own = static_cast<uint8_t*>(peers->regions[peers->rank]);
  if (!own) return MOSAIC_ERR_SHAPE;
  const EpPeersDev d = ep_dev(peers);
  if (recv_rows) *recv_rows = own + d.recv_off;
  if (recv_count) *recv_count = &reinterpret_cast<EpRegionHeader*>(own)->recv_count;
  if (ret_partials) *ret_partials = own + d.ret_off;
  return MOSAIC_OK;
}

int mosaic_ep_exchange_rows(const mosaic_ep_peers* peers, const void* send_rows, const int32_t* dest_counts,
                            mosaic_stream_t stream) {
  int st = check_peers(peers);
  if (st) return st;
  st = check_regions(peers);
  if (st) return st;
  if (!send_rows || !dest_counts) return MOSAIC_ERR_SHAPE;
  if (!aligned(send_rows, 16) || !aligned(dest_counts, 4)) return MOSAIC_ERR_ALIGN;
  const int sms = sm_count();
  if (sms <= 0) return MOSAIC_ERR_CUDA;
  return launch_ep_exchange_rows(ep_dev(peers), send_rows, dest_counts, sms, reinterpret_cast<cudaStream_t>(stream)) ==
                 cudaSuccess
             ? MOSAIC_OK
             : MOSAIC_ERR_CUDA;
}

size_t mosaic_ep_expert_rows_workspace_bytes(const mosaic_moe_dims* dims, const mosaic_ep_peers* peers) {
  if (!dims || check_peers(peers) != MOSAIC_OK) return 0;
  if (!peers->unit_slots) return mosaic_moe_expert_rows_workspace_bytes(dims, peers->max_recv_rows);
  if (dims->n_experts > 256) return 0;
  const mosaic_moe_dims r = units_dims(dims, peers);
  if (check_rows_dims(&r) != MOSAIC_OK) return 0;
  return units_ws(&r).total;
}

int mosaic_ep_expert_rows_return(const mosaic_moe_dims* dims, const mosaic_ep_peers* peers,
                                 const mosaic_expert_bank* bank, void* workspace, size_t workspace_bytes,
                                 mosaic_stream_t stream) {
  int st = check_peers(peers);
  if (st) return st;
  st = check_regions(peers);
  if (st) return st;
  if (!dims) return MOSAIC_ERR_SHAPE;
  if (dims->hidden != peers->hidden || (dims->act_mode == MOSAIC_ACT_BF16) != (peers->partial_f32 != 0))
    return MOSAIC_ERR_SHAPE;
  const EpPeersDev ep = ep_dev(peers);
  uint8_t* own = static_cast<uint8_t*>(peers->regions[peers->rank]);
  uint8_t* recv = own + ep.recv_off;
  const int32_t* count = &reinterpret_cast<EpRegionHeader*>(own)->recv_count;
  const int rb = ep.row_bytes;
  const int h = peers->hidden;
  const bool e4m3 = peers->row_e4m3 != 0;
  if (peers->unit_slots) {  // unit rows: expand every unit into its slots' packed rows
    if (dims->act_mode != MOSAIC_ACT_FP8 || dims->n_experts > 256) return MOSAIC_ERR_SHAPE;
    const mosaic_moe_dims r = units_dims(dims, peers);
    st = check_rows_dims(&r);
    if (st) return st;
    st = check_bank(bank);
    if (st) return st;
    if (!workspace) return MOSAIC_ERR_SHAPE;
    if (!aligned(workspace, 256)) return MOSAIC_ERR_ALIGN;
    const UnitsWs uw = units_ws(&r);
    if (workspace_bytes < uw.total) return MOSAIC_ERR_WORKSPACE;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    const WsPlan& w = uw.plan;
    if (cudaMemsetAsync(ws + w.err, 0, 16, s) != cudaSuccess) return MOSAIC_ERR_CUDA;
    const int K = peers->unit_slots, U = peers->max_recv_rows;
    int64_t* aidx = reinterpret_cast<int64_t*>(ws + uw.idx);
    float* aw = reinterpret_cast<float*>(ws + uw.w);
    int* arank = reinterpret_cast<int*>(ws + uw.a_rank);
    int* apos = reinterpret_cast<int*>(ws + uw.a_pos);
    int* rrank = reinterpret_cast<int*>(ws + uw.row_rank);
    int* rret = reinterpret_cast<int*>(ws + uw.row_ret);
    if (launch_ep_units_meta(ep, h, K, U, aidx, aw, arank, apos, s) != cudaSuccess) return MOSAIC_ERR_CUDA;
    LayoutParams lp{};
    lp.idx = aidx;
    lp.weights = aw;
    lp.T = U;
    lp.k = K;
    lp.E = r.n_experts;
    lp.with_shared = 0;
    fill_layout(lp, w, ws);
    lp.T_dev = count;
    lp.row_sorted = nullptr;
    lp.pad_ok = 1;  // unused slots
    if (launch_layout(lp, s) != cudaSuccess) return MOSAIC_ERR_CUDA;
    if (launch_rows_place_units(recv, rb, U, count, h, K, lp.row_of, arank, apos, w.R_pad, lp.row_tile, lp.row_pos,
                                ws + w.xq, reinterpret_cast<uint32_t*>(ws + w.x_sft), rrank, rret, s) != cudaSuccess)
      return MOSAIC_ERR_CUDA;
    st = run_gemms(&r, w, ws, lp, bank, dims->has_shared ? dims->n_experts : -1, lp.row_token, nullptr, s, nullptr,
                   &ep, nullptr, 0, rrank, rret);
    if (st) return st;
    return launch_ep_signal_return(ep, s) == cudaSuccess ? MOSAIC_OK : MOSAIC_ERR_CUDA;
  }
  const int meta = e4m3 ? rb - 16 : 2 * h;  // byte offset of the row's tail
  st = expert_rows_impl(dims, peers->max_recv_rows, count, recv, e4m3 ? rb : rb / 2,
                        reinterpret_cast<const int32_t*>(recv + meta), reinterpret_cast<const float*>(recv + meta + 4),
                        rb / 4, 0, bank, nullptr, workspace, workspace_bytes, stream, &ep, e4m3 ? rb : 0);
  if (st) return st;
  return launch_ep_signal_return(ep, reinterpret_cast<cudaStream_t>(stream)) == cudaSuccess ? MOSAIC_OK
                                                                                          : MOSAIC_ERR_CUDA;
}

int mosaic_ep_return_partials(const mosaic_ep_peers* peers, const void* partials, mosaic_stream_t stream) {
  int st = check_peers(peers);
  if (st) return st;
  st = check_regions(peers);
  if (st) return st;
  if (!partials) return MOSAIC_ERR_SHAPE;
  if (!aligned(partials, 16)) return MOSAIC_ERR_ALIGN;
  const int sms = sm_count();
  if (sms <= 0) return MOSAIC_ERR_CUDA;
  return launch_ep_return_partials(ep_dev(peers), partials, sms, reinterpret_cast<cudaStream_t>(stream)) ==
                 cudaSuccess
             ? MOSAIC_OK
             : MOSAIC_ERR_CUDA;
}

int mosaic_ep_dispatch_exchange(const mosaic_moe_dims* dims, const mosaic_ep_peers* peers, const void* x,
                                const int64_t* idx, const float* weights, void* workspace, size_t workspace_bytes,
                                mosaic_stream_t stream) {
  int st = check_dims(dims);
  if (st) return st;
  st = check_peers(peers);
  if (st) return st;
  st = check_regions(peers);
  if (st) return st;
  if (!x || !idx || !workspace) return MOSAIC_ERR_SHAPE;
  if (!peers->row_e4m3 || dims->act_mode != MOSAIC_ACT_FP8 || dims->hidden != peers->hidden) return MOSAIC_ERR_SHAPE;
  const int world = peers->world;
  if (dims->n_experts % world) return MOSAIC_ERR_SHAPE;
  if (dims->tokens > peers->max_tokens ||
      static_cast<int64_t>(dims->tokens) * dims->top_k > static_cast<int64_t>(peers->max_send_rows))
    return MOSAIC_ERR_SHAPE;
  if (!aligned(x, 16) || !aligned(idx, 8) || (weights && !aligned(weights, 4)) || !aligned(workspace, 256))
    return MOSAIC_ERR_ALIGN;
  const WsPlan w = plan_ws(dims);
  if (workspace_bytes < w.total) return MOSAIC_ERR_WORKSPACE;
  const int sms = sm_count();
  if (sms <= 0) return MOSAIC_ERR_CUDA;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  if (cudaMemsetAsync(ws + w.err, 0, 16, s) != cudaSuccess) return MOSAIC_ERR_CUDA;
  const int T = dims->tokens, k = dims->top_k, E = dims->n_experts;
  LayoutParams lp{};
  lp.idx = idx;
  lp.weights = weights;
  lp.T = T;
  lp.k = k;
  lp.E = E;
  lp.with_shared = 0;
  fill_layout(lp, w, ws);
  lp.row_tile = nullptr;  // no GEMM tiles on the sending side
  lp.row_pos = nullptr;
  lp.tiles = nullptr;
  if (launch_layout(lp, s) != cudaSuccess) return MOSAIC_ERR_CUDA;
  // the sender runs no GEMM, so the activation planes and the partial rows of
  // the workspace are free: the destination counts (and, with unit rows, the
  // units' tokens [world][T]) and the E4M3 token rows (T x (H + pad) <= T x 2H
  // bytes of the R x H partials)
  int* dest_counts = reinterpret_cast<int*>(ws + w.xq);
  if (peers->unit_slots) {
    const int E_local = E / world;
    if (peers->unit_slots < (k < E_local ? k : E_local)) return MOSAIC_ERR_SHAPE;
    int* unit_token = reinterpret_cast<int*>(ws + w.xq + 256);
    if (launch_ep_dispatch_send_units(ep_dev(peers), x, T, dims->hidden, k, E_local, peers->unit_slots, idx,
                                      weights, lp.row_of, dest_counts, unit_token, ws + w.partial, sms,
                                      s) != cudaSuccess)
      return MOSAIC_ERR_CUDA;
    return MOSAIC_OK;
  }
  if (launch_ep_dispatch_send_e4m3(ep_dev(peers), x, T, dims->hidden, E, E / world, lp.offsets, lp.row_token,
                                   lp.row_weight, dest_counts, ws + w.partial, sms, s) != cudaSuccess)
    return MOSAIC_ERR_CUDA;
  return MOSAIC_OK;
}

int mosaic_ep_combine(const mosaic_moe_dims* dims, const void* partials, const void* workspace, void* y,
                      mosaic_stream_t stream) {
  int st = check_dims(dims);
  if (st) return st;
  if (!partials || !workspace || !y) return MOSAIC_ERR_SHAPE;
  if (!aligned(partials, 16) || !aligned(y, 16) || !aligned(workspace, 256)) return MOSAIC_ERR_ALIGN;
  const WsPlan w = plan_ws(dims);
  const uint8_t* ws = static_cast<const uint8_t*>(workspace);
  const int T = dims->tokens, k = dims->top_k;
  if (launch_combine(partials, w.partial_f32, reinterpret_cast<const int*>(ws + w.row_sorted), T, k, dims->hidden,
                     dims->has_shared ? T * k : -1, y, reinterpret_cast<cudaStream_t>(stream)) != cudaSuccess)
    return MOSAIC_ERR_CUDA;
  return MOSAIC_OK;
}

int mosaic_read_error(const void* workspace, int32_t reset, int32_t* code_out, mosaic_stream_t stream) {
  if (!workspace || !code_out) return MOSAIC_ERR_SHAPE;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int32_t v = 0;
  if (cudaMemcpyAsync(&v, workspace, sizeof(v), cudaMemcpyDeviceToHost, s) != cudaSuccess) return MOSAIC_ERR_CUDA;
  if (cudaStreamSynchronize(s) != cudaSuccess) return MOSAIC_ERR_CUDA;
  if (reset && cudaMemsetAsync(const_cast<void*>(workspace), 0, 16, s) != cudaSuccess) return MOSAIC_ERR_CUDA;
  *code_out = v;
  return MOSAIC_OK;
}

}  // extern "C"
