// Grouped block-scaled expert GEMM for the MoE layer (tcgen05, sm_100a).
//
// One persistent kernel serves both expert projections:
//   mode 0 (gate/up): D_gate = W_gate . X^T and D_up = W_up . X^T for a 128-row
//     block of the intermediate dimension, then the epilogue computes
//     z = SiLU(clamp(gate)) * clamp(up) * route_weight, rounds z to bf16 and
//     re-quantises it (FP8 mode: the reference act_quant per 128; bf16 mode:
//     hi + lo E4M3 with per-32 scales) straight into the down GEMM's input
//     rows and scale-factor chunks;
//   mode 1 (down): D = W_down . Z^T for a 128-row block of the hidden
//     dimension, written as per-assignment partials (fp32 or bf16).
//
// Swap-AB orientation: A = expert weights (E2M1 codes, E8M0 per-32 scales;
// MMA M = 128 weight rows), B = the activation rows of one token tile of one
// expert (E4M3, per-32 scales; MMA N = token rows padded to 16, doubled in
// bf16 mode for the lo plane).
//
// Data movement is shaped for the TMA unit, whose per-operation cost dominates
// at decode sizes: every stage moves its 16 KB of packed weights with ONE
// tensor load (gate + up tiles of one K-tile are adjacent in the bank, and the
// down GEMM takes two consecutive K-tiles per stage), unpacked by the
// 16U4_ALIGN16B type into the smem layout kind::mxf8f6f4 reads.  A dedicated
// warp issues only those loads; a second producer warp issues the activation
// rows (one 4-D box: K-tiles x planes x rows) and the scale-factor chunks.
// Scale factors go smem -> TMEM with tcgen05.cp; accumulators live in TMEM,
// double-buffered with independent K chains at decode sizes.
//
// Warp roles (320 threads): warp 0 = weight producer, warp 6 = activation /
// scale producer, warps 2..5 = epilogue (warp w reads TMEM lanes 32*(w%4)..+31),
// warps 1, 7, 8, 9 = MMA issuers (warp 1 also owns TMEM).  A tcgen05.mma costs
// its issuing thread ~150-200 cycles whatever its size, so a single issuer
// caps small-N decode tiles far below HBM speed; four issuers split every
// stage into two units (gate / up, or the two K-tiles of a down stage) and
// alternate stages by parity, each accumulating into its own TMEM chain with
// its own scale-factor columns.  The epilogue sums the chains in a fixed order.
// Reference behaviour: mosaicvm/kernels/qpa_mma.py:337-486 (grouped ordered
// gate/up and down kernels), mosaicvm/kernels/mxint.py:1301-1346 (fused
// SwiGLU / route weight / bf16 / act_quant epilogue).
#include "common.cuh"
#include "kernels.h"

namespace mosaic {

namespace {

constexpr int kThreads = 320;
constexpr uint32_t kTmemCols = 512;
constexpr int kMaxStages = 8;
constexpr int kSmemBudget = 225 * 1024;

struct Ctrl {
  uint64_t full[kMaxStages];
  uint64_t empty[kMaxStages];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t drain[4];
  uint32_t tmem_base;
  int abort;
  float red[4][16];
};

// Per stage: two 16 KB weight tiles (gate+up of one K-tile, or two K-tiles of
// down), KS activation sub-tiles of planes x brows rows, two weight scale
// chunks and KS activation scale chunks.
struct Plan {
  int stage_bytes, off_b, b_sub, off_sfa, off_sfb, stages, ks;
};

__host__ __device__ inline Plan make_plan(int mode, int planes, int brows, int ks) {
  Plan pl;
  pl.ks = (mode == 0) ? 1 : ks;
  pl.b_sub = planes * brows * 128;
  pl.off_b = 32768;
  pl.off_sfa = pl.off_b + ((pl.ks * pl.b_sub + 1023) / 1024) * 1024;
  pl.off_sfb = pl.off_sfa + 1024;
  pl.stage_bytes = ((pl.off_sfb + 512 * pl.ks + 1023) / 1024) * 1024;
  int s = (kSmemBudget - static_cast<int>(sizeof(Ctrl)) - 1024) / pl.stage_bytes;
  pl.stages = s > kMaxStages ? kMaxStages : s;
  return pl;
}

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// 4-D tensor load (activation rows: {128 B, rows, planes, K-tiles}).
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2,
                                            int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// Sum over the C accumulation chains (chain stride acc_w columns) of 16 columns,
// adding the lo-plane columns (lo_off > 0: columns lo_off.. of the same chain).
// Chains and planes are added in a fixed order, so the result is deterministic.
__device__ __forceinline__ void tmem_sum16(uint32_t taddr, int C, uint32_t acc_w, int lo_off, float (&out)[16]) {
#pragma unroll
  for (int j = 0; j < 16; ++j) out[j] = 0.f;
  for (int c = 0; c < C; ++c) {
    uint32_t r[16], r2[16];
    tmem_ld16(taddr + c * acc_w, r);
    if (lo_off) tmem_ld16(taddr + c * acc_w + lo_off, r2);
    tmem_ld_wait();
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      float v = __uint_as_float(r[j]);
      if (lo_off) v += __uint_as_float(r2[j]);
      out[j] += v;
    }
  }
}

// Word index, inside a 512-byte scale chunk, of token row n (< 128).
__device__ __forceinline__ int sf_word(int n) { return (n & 31) * 4 + (n >> 5); }

struct Item {
  int tile, nb, e, row0, rows, rpad, n;
};

__device__ __forceinline__ Item get_item(const GemmParams& p, int item) {
  Item it;
  it.tile = item / p.n_blocks;
  it.nb = item - it.tile * p.n_blocks;
  it.e = p.tiles[3 * it.tile + 0];
  it.row0 = p.tiles[3 * it.tile + 1];
  it.rows = p.tiles[3 * it.tile + 2];
  it.rpad = (it.rows + 15) & ~15;
  it.n = p.hilo ? 2 * it.rpad : it.rpad;
  return it;
}

__global__ void __launch_bounds__(kThreads, 1)
    moe_gemm_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                    const GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int planes = p.hilo ? 2 : 1;
  const Plan pl = make_plan(p.mode, planes, p.brows, p.ks);
  const int S = pl.stages;
  const int KS = pl.ks;
  Ctrl* ctrl = reinterpret_cast<Ctrl*>(smem + S * pl.stage_bytes);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const bool gu = (p.mode == 0);
  const int nbuf = p.nbuf;
  const int P = p.parities;  // stage parities split across issuer pairs (1 or 2)
  // TMEM: accumulator of (buffer b, chain c) at column (b*CH + c) * acc_w with
  // CH = P chains (gate/up: the up half at +max_n) or P*KS chains (down: chain
  // p*KS + u).  Issuer i's scale factors: weight chunk at sf_base + 8i, token
  // chunk at +4.
  const uint32_t acc_w = static_cast<uint32_t>((gu ? 2 : 1) * p.max_n);
  const uint32_t up_off = static_cast<uint32_t>(p.max_n);
  const int CH = gu ? P : P * KS;
  const uint32_t sf_base = kTmemCols - 32u;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&ctrl->full[s], 2);   // one arrival from each producer warp
      mbar_init(&ctrl->empty[s], 4);  // every issuer: a commit (consumer) or an arrive (observer)
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&ctrl->acc_full[b], 4);  // one commit from each issuer
      mbar_init(&ctrl->acc_empty[b], 128);
    }
    for (int i = 0; i < 4; ++i) mbar_init(&ctrl->drain[i], 1);
    ctrl->abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) prefetch_tmap(&tmap_w);
  if (warp == 6 && lane == 0) prefetch_tmap(&tmap_x);
  if (warp == 1) {
    tmem_alloc(&ctrl->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctrl->tmem_base;
  volatile int* abort = &ctrl->abort;

  int n_tiles = *p.n_tiles;
  if (n_tiles > p.max_tiles) n_tiles = p.max_tiles;
  const int n_items = n_tiles * p.n_blocks;
  const int KT = p.K / 128;
  const int n_stages_item = KT / KS;

  if (warp == 0 || warp == 6) {
    // ----------------------------------------------------------- producers
    const bool wprod = (warp == 0);
    int it = 0;
    bool ok = true;
    for (int item = blockIdx.x; ok && item < n_items; item += gridDim.x) {
      const Item m = get_item(p, item);
      // weight tile index of (expert, row block, K-tile 0); the tiles of one K-tile
      // are [gate, up] in mode 0, and consecutive K-tiles follow each other
      const int wtile = ((m.e * p.n_blocks + m.nb) * KT) * (gu ? 2 : 1);
      // The weight warp issues exactly one TMA per stage (the TMA unit's per-op
      // cost, not bytes, limits a single issuing thread); everything small -
      // activation rows and all scale-factor chunks - comes from warp 6.
      const uint32_t wtiles = gu ? 2u : static_cast<uint32_t>(KS);  // 8 KB tiles per weight box
      const uint32_t tx = wprod ? wtiles * 8192u
                                : wtiles * 512u +
                                      static_cast<uint32_t>(KS) * (static_cast<uint32_t>(planes * p.brows) * 128u + 512u);
      for (int ks = 0; ks < n_stages_item; ++ks, ++it) {
        const int s = it % S;
        const uint32_t ph = static_cast<uint32_t>(it / S) & 1u;
        if (!mbar_wait(&ctrl->empty[s], ph ^ 1u, abort)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          uint8_t* st = smem + s * pl.stage_bytes;
          uint64_t* fb = &ctrl->full[s];
          const int kt = ks * KS;
          // gate+up of K-tile kt (mode 0) or K-tiles kt.. kt+KS-1 (mode 1)
          const int t0 = wtile + kt * (gu ? 2 : 1);
          mbar_arrive_expect_tx(fb, tx);
          if (wprod) {
            tma_load_3d(st, &tmap_w, fb, 0, 0, t0);
          } else {
            tma_load_4d(st + pl.off_b, &tmap_x, fb, 0, m.row0, 0, kt);
            bulk_load(st + pl.off_sfa, p.w_sf + static_cast<size_t>(t0) * 512, 512u * wtiles, fb);
            bulk_load(st + pl.off_sfb, p.x_sft + (static_cast<size_t>(m.tile) * KT + kt) * 512, 512 * KS, fb);
          }
        }
        __syncwarp();
      }
    }
    if (!ok) {
      if (lane == 0) set_error(p.err, MOSAIC_ERR_TIMEOUT);
      ctrl->abort = 1;
    }
    // Wait (bounded) for the last armed stage so no copy is in flight at exit.
    if (it > 0 && lane == 0) {
      const int s = (it - 1) % S;
      volatile int never = 0;
      mbar_wait(&ctrl->full[s], static_cast<uint32_t>((it - 1) / S) & 1u, &never);
    }
    __syncwarp();
  } else if (warp == 1 || warp >= 7) {
    // ----------------------------------------------------------------- MMA
    const int issuer = (warp == 1) ? 0 : warp - 6;  // 0..3
    const int ip = issuer >> 1;                     // stage parity this issuer takes
    const int iu = issuer & 1;                      // unit: gate/up half, or down K sub-tile
    const uint32_t col_sfw = tmem + sf_base + 8u * issuer;  // weight scale chunk
    const uint32_t col_sfx = col_sfw + 4u;                  // token scale chunk
    int it = 0, li = 0;
    bool issued = false, ok = true;
    for (int item = blockIdx.x; ok && item < n_items; item += gridDim.x, ++li) {
      const Item m = get_item(p, item);
      const int b = li % nbuf;
      const uint32_t aph = static_cast<uint32_t>(li / nbuf) & 1u;
      if (!mbar_wait(&ctrl->acc_empty[b], aph ^ 1u, abort)) {
        ok = false;
        break;
      }
      tc_fence_after();
      for (int ks = 0; ks < n_stages_item; ++ks, ++it) {
        const int s = it % S;
        const uint32_t ph = static_cast<uint32_t>(it / S) & 1u;
        // Every issuer observes every phase of every full barrier and arrives on
        // the matching empty barrier, including for the stages the other parity
        // consumes.  A parity wait that skipped phases could match the phase two
        // fills back and read a stage before it lands; requiring every issuer's
        // arrival before a refill keeps all four within one phase of the ring.
        if (!mbar_wait(&ctrl->full[s], ph, abort)) {
          ok = false;
          break;
        }
        if (ks % P != ip) {
          if (lane == 0) mbar_arrive(&ctrl->empty[s]);
          __syncwarp();
          continue;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t sw = smem_u32(smem + s * pl.stage_bytes);
          const bool first = (ks < P);  // first stage of this issuer's chain in the item
          if (gu) {
            const uint32_t d = tmem + static_cast<uint32_t>(b * CH + ip) * acc_w + (iu ? up_off : 0u);
            tc_cp_32x128b_x4(col_sfw, desc_sf(sw + pl.off_sfa + 512 * iu));
            tc_cp_32x128b_x4(col_sfx, desc_sf(sw + pl.off_sfb));
            const uint32_t a = sw + 16384 * iu, bb = sw + pl.off_b;
#pragma unroll
            for (uint32_t kb = 0; kb < 4; ++kb) {
              tc_mma_mxf8f6f4(d, desc_sw128(a + kb * 32), desc_sw128(bb + kb * 32), idesc_mxf8f6f4(m.n, kb),
                              (first && kb == 0) ? 0u : 1u, col_sfw | (kb << 30), col_sfx | (kb << 30));
            }
          } else if (iu < KS) {
            const uint32_t d = tmem + static_cast<uint32_t>(b * CH + ip * KS + iu) * acc_w;
            tc_cp_32x128b_x4(col_sfw, desc_sf(sw + pl.off_sfa + 512 * iu));
            tc_cp_32x128b_x4(col_sfx, desc_sf(sw + pl.off_sfb + 512 * iu));
            const uint32_t a = sw + 16384 * iu, bb = sw + pl.off_b + pl.b_sub * iu;
#pragma unroll
            for (uint32_t kb = 0; kb < 4; ++kb) {
              tc_mma_mxf8f6f4(d, desc_sw128(a + kb * 32), desc_sw128(bb + kb * 32), idesc_mxf8f6f4(m.n, kb),
                              (first && kb == 0) ? 0u : 1u, col_sfw | (kb << 30), col_sfx | (kb << 30));
            }
          }
          tc_commit(&ctrl->empty[s]);  // a unit without work still arrives
          issued = true;
        }
        __syncwarp();
      }
      if (!ok) break;
      if (lane == 0) {
        tc_commit(&ctrl->acc_full[b]);
        issued = true;
      }
      __syncwarp();
    }
    if (!ok) {
      if (lane == 0) set_error(p.err, MOSAIC_ERR_TIMEOUT);
      ctrl->abort = 1;
    }
    // Drain: every MMA / copy this warp issued has completed before TMEM is freed.
    if (lane == 0 && issued) {
      tc_commit(&ctrl->drain[issuer]);
      volatile int never = 0;
      mbar_wait(&ctrl->drain[issuer], 0, &never);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int lrow = q * 32 + lane;
    const uint32_t tq = tmem + (static_cast<uint32_t>(q * 32) << 16);
    const size_t z_plane = static_cast<size_t>(p.R_pad) * 128;    // bytes per (K-tile, plane) of z rows
    const size_t z_ktile = static_cast<size_t>(planes) * z_plane;  // bytes per K-tile of z rows
    int li = 0;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x, ++li) {
      const Item m = get_item(p, item);
      const bool round_mid = p.fp8 || (m.e == p.shared_expert);
      const int b = li % nbuf;
      const uint32_t aph = static_cast<uint32_t>(li / nbuf) & 1u;
      if (!mbar_wait(&ctrl->acc_full[b], aph, abort)) {
        if (lane == 0) set_error(p.err, MOSAIC_ERR_TIMEOUT);
        ctrl->abort = 1;
        break;
      }
      tc_fence_after();
      const uint32_t c_buf = static_cast<uint32_t>(b * CH) * acc_w;
      const int P_used = n_stages_item < P ? n_stages_item : P;  // chains that received MMAs
      const int C = gu ? P_used : P_used * KS;
      for (int c0 = 0; c0 < m.rpad; c0 += 16) {
        if (gu) {
          float gs[16], us[16];
          tmem_sum16(tq + c_buf + c0, C, acc_w, p.hilo ? m.rpad : 0, gs);
          tmem_sum16(tq + c_buf + up_off + c0, C, acc_w, p.hilo ? m.rpad : 0, us);
          float zd[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int col = c0 + j;
            float gv = gs[j];
            float uv = us[j];
            if (round_mid) {
              gv = bf16r(gv);
              uv = bf16r(uv);
            }
            if (p.swiglu_limit > 0.f) {
              gv = fminf(gv, p.swiglu_limit);
              uv = fminf(fmaxf(uv, -p.swiglu_limit), p.swiglu_limit);
            }
            const float w = (col < m.rows) ? p.row_weight[m.row0 + col] : 0.f;
            float z = gv / (1.0f + expf(-gv)) * uv;
            z = z * w;
            zd[j] = (col < m.rows) ? bf16r(z) : 0.f;
          }
          // z rows: [K-tile = nb][plane][row][128 B]; this thread owns byte lrow of the K-tile
          uint8_t* zq = p.zq + static_cast<size_t>(m.nb) * z_ktile + lrow;
          uint32_t* zsf = p.z_sft + (static_cast<size_t>(m.tile) * (p.I / 128) + m.nb) * 128;
          if (p.fp8) {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const float mx = warp_max(fabsf(zd[j]));
              if (lane == 0) ctrl->red[q][j] = mx;
            }
            epi_bar();
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int col = c0 + j;
              const float amax =
                  fmaxf(fmaxf(ctrl->red[0][j], ctrl->red[1][j]), fmaxf(ctrl->red[2][j], ctrl->red[3][j]));
              const int ex = pow2_scale_exp(amax, 1e-4f);
              const float y = fminf(fmaxf(zd[j] * exp2i(-ex), -448.f), 448.f);
              if (col < m.rows) {
                zq[static_cast<size_t>(m.row0 + col) * 128] = f32_to_e4m3(y);
                if (lrow == 0) zsf[sf_word(col)] = (static_cast<uint32_t>(ex + 127) & 0xFFu) * 0x01010101u;
              }
            }
            epi_bar();
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int col = c0 + j;
              const float mx = warp_max(fabsf(zd[j]));
              int eh = pow2_scale_exp(mx, 1e-30f);
              eh = max(-126, min(127, eh));
              const uint8_t hb = f32_to_e4m3(zd[j] * exp2i(-eh));
              const float res = zd[j] - e4m3_to_f32(hb) * exp2i(eh);
              const float m2 = warp_max(fabsf(res));
              int el = pow2_scale_exp(m2, fmaxf(mx * 1e-7f, 1e-30f));
              el = max(-126, min(127, el));
              const uint8_t lb = f32_to_e4m3(res * exp2i(-el));
              if (col < m.rows) {
                const size_t r = static_cast<size_t>(m.row0 + col) * 128;
                zq[r] = hb;
                zq[z_plane + r] = lb;
                if (lane == 0) {
                  reinterpret_cast<uint8_t*>(zsf + sf_word(col))[q] = static_cast<uint8_t>(eh + 127);
                  reinterpret_cast<uint8_t*>(zsf + sf_word(m.rpad + col))[q] = static_cast<uint8_t>(el + 127);
                }
              }
            }
          }
        } else {
          float ds[16];
          tmem_sum16(tq + c_buf + c0, C, acc_w, p.hilo ? m.rpad : 0, ds);
          const int nn = m.nb * 128 + lrow;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int col = c0 + j;
            if (col < m.rows) {
              float v = ds[j];
              if (round_mid) v = bf16r(v);
              const int orow = p.out_row ? p.out_row[m.row0 + col] : m.row0 + col;
              const size_t o = static_cast<size_t>(orow) * p.H + nn;
              if (p.out_f32)
                reinterpret_cast<float*>(p.out)[o] = v;
              else
                reinterpret_cast<__nv_bfloat16*>(p.out)[o] = __float2bfloat16_rn(v);
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&ctrl->acc_empty[b]);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

}  // namespace

size_t gemm_smem_bytes(int mode, int planes, int brows, int ks) {
  const Plan pl = make_plan(mode, planes, brows, ks);
  return static_cast<size_t>(pl.stages) * pl.stage_bytes + sizeof(Ctrl) + 1024;
}

cudaError_t launch_moe_gemm(const CUtensorMap& tmap_w, const CUtensorMap& tmap_x, const GemmParams& p, int grid,
                            cudaStream_t stream) {
  if (p.max_n < 16 || p.max_n > 128 || p.nbuf < 1 || p.nbuf > 2 || p.parities < 1 || p.parities > 2)
    return cudaErrorInvalidValue;
  const int planes = p.hilo ? 2 : 1;
  if (p.brows * planes != p.max_n || p.brows % 16) return cudaErrorInvalidValue;
  const int acc_w = (p.mode == 0 ? 2 : 1) * p.max_n;
  const int ch = (p.mode == 0) ? p.parities : p.parities * p.ks;
  if (p.nbuf * ch * acc_w > static_cast<int>(kTmemCols) - 32) return cudaErrorInvalidValue;
  const int KT = p.K / 128;
  if (p.ks < 1 || p.ks > 2 || (p.mode == 0 && p.ks != 1)) return cudaErrorInvalidValue;
  if (KT % p.ks) return cudaErrorInvalidValue;
  const Plan pl = make_plan(p.mode, planes, p.brows, p.ks);
  if (pl.stages < 2) return cudaErrorInvalidValue;
  const size_t smem = gemm_smem_bytes(p.mode, planes, p.brows, p.ks);
  cudaError_t err = cudaFuncSetAttribute(moe_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
  if (err != cudaSuccess) return err;
  moe_gemm_kernel<<<grid, kThreads, smem, stream>>>(tmap_w, tmap_x, p);
  return cudaGetLastError();
}

}  // namespace mosaic
