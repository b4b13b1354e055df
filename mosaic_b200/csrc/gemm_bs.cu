// Grouped block-scaled expert GEMM for the MoE layer (tcgen05, sm_100a).
//
// One persistent kernel serves both expert projections.  A work item is one
// token tile of one expert times a PAIR of 128-row weight blocks, which share
// the item's activation tile:
//   mode 0 (gate/up): the gate block and the up block of 128 intermediate
//     rows; the epilogue computes z = SiLU(clamp(gate)) * clamp(up) *
//     route_weight, rounds z to bf16 and re-quantises it (FP8 mode: the
//     reference act_quant per 128; bf16 mode: hi + lo E4M3 with per-32
//     scales) straight into the down GEMM's input rows and scale chunks;
//   mode 1 (down): hidden rows [nb*128, +128) and [H/2 + nb*128, +128); the
//     epilogue writes per-assignment partials (fp32 or bf16).
// The bank keeps the two tiles of a pair adjacent for every K-tile (the
// "halves" re-layout), so one tensor load moves both.
//
// Swap-AB orientation: A = expert weights (E2M1 codes, E8M0 per-32 scales;
// MMA M = 128 weight rows), B = the activation rows of one token tile of one
// expert (E4M3, per-32 scales; MMA N = token rows padded to 16, doubled in
// bf16 mode for the lo plane).
//
// Data movement: every stage moves its 16 KB of packed weights with ONE
// tensor load, unpacked by the 16U4_ALIGN16B type into the smem layout
// kind::mxf8f6f4 reads, from a warp that issues nothing else; a second
// producer warp issues the activation K-tile (one 4-D box: planes x rows) and
// the scale-factor chunks.  Scale factors go smem -> TMEM with tcgen05.cp;
// accumulators live in TMEM, double-buffered, so the epilogue of one item
// overlaps the MMAs of the next.  The epilogue stages its output in shared
// memory and writes whole token rows with 16-byte stores.
//
// Warp roles (416 threads): warp 0 = weight producer, warp 6 = activation /
// scale producer, warp 12 = scale-factor copier (tcgen05.cp of each stage's
// weight and token scale chunks into a TMEM ring, one slot per smem stage;
// the 384-thread instance for single-buffered launches has no copier and the
// issuers copy their own chunks),
// warps 2..5 = epilogue (warp w reads TMEM lanes 32*(w%4)..+31),
// warps 1, 7..11 = up to three pairs of MMA issuers (warp 1 also owns TMEM).  A
// tcgen05.mma costs its issuing thread ~150-200 cycles whatever its size, so
// each stage is split into two units (the two blocks of the pair), and at
// decode sizes three issuer pairs take the stages in turn (stage parity modulo
// 3), each accumulating into its own TMEM chain.  The copier keeps the scale
// copies off the issuers (a copy costs its issuing thread about a quarter of
// an MMA).  The epilogue sums the chains in a fixed order.
// With an expert slot table the producers read logical expert e's weights and
// scales from bank entry expert_slot[e] (an offload cache); everything else
// uses the logical id, so results do not depend on where the expert sits.
// Reference behaviour: mosaicvm/kernels/qpa_mma.py:337-486 (grouped ordered
// gate/up and down kernels), mosaicvm/kernels/mxint.py:1301-1346 (fused
// SwiGLU / route weight / bf16 / act_quant epilogue).
#include "common.cuh"
#include "kernels.h"

namespace mosaic {

namespace {

constexpr int kThreadsCopier = 416;  // 13 warps: + warp 12, the scale-factor copier (128 registers)
constexpr int kThreadsPlain = 384;   // 12 warps: issuers copy their own scale chunks (up to 168 registers)
constexpr uint32_t kTmemCols = 512;
constexpr int kMaxStages = 8;
constexpr int kSmemBudget = 225 * 1024;
constexpr int kEpiBytes = 16 * 256 * 4;  // epilogue staging: 16 token columns x 256 values (fp32)
constexpr int kMaxParities = 3;          // issuer pairs (two MMA warps each)
constexpr uint32_t kSfSlotCols = 12u;  // copier: TMEM scale columns per ring stage (2 weight chunks + token)
constexpr uint32_t kSfIssuerCols = 8u * 2 * kMaxParities;  // no copier: 8 columns per issuer

struct Ctrl {
  uint64_t full[kMaxStages];
  uint64_t empty[kMaxStages];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t drain[7];
  uint64_t sf_ready[kMaxStages];
  uint32_t tmem_base;
  int abort;
  // per epilogue group (two in the E4M3 instance, one otherwise):
  float4 red4[2][2][16];  // gate/up act_quant: column maxima of the group's four warps, two blocks
  float meta_w[2][128];   // gate/up: route weight of each row of the item's token tile
  int meta_o[2][128];     // down: output row (EP: row in the source's return buffer)
  int meta_r[2][128];     // down, EP: source rank of the row
};

// Per stage: the two 16 KB (unpacked) weight tiles of the pair for one
// K-tile, the activation K-tile (planes x brows rows of 128 B), the pair's two
// weight scale chunks and the token tile's scale chunk.
struct Plan {
  int stage_bytes, off_b, off_sfa, off_sfb, stages, epi;
};

__host__ __device__ constexpr Plan make_plan(int planes, int brows) {
  Plan pl{};
  pl.off_b = 32768;
  pl.off_sfa = pl.off_b + ((planes * brows * 128 + 1023) / 1024) * 1024;
  pl.off_sfb = pl.off_sfa + 1024;
  pl.stage_bytes = ((pl.off_sfb + 512 + 1023) / 1024) * 1024;
  int s = (kSmemBudget - static_cast<int>(sizeof(Ctrl)) - kEpiBytes - 1024) / pl.stage_bytes;
  pl.stages = s > kMaxStages ? kMaxStages : s;
  pl.epi = pl.stages * pl.stage_bytes;  // epilogue staging right after the ring (1 KB aligned)
  return pl;
}

// Named barrier (1 + g) of epilogue group g's four warps.
__device__ __forceinline__ void epi_bar(int g) { asm volatile("bar.sync %0, 128;" ::"r"(1 + g) : "memory"); }
// The same barrier, also ANDing a predicate over the group.
__device__ __forceinline__ bool epi_all(int g, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.and.pred q, %2, 128, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(v)), "r"(1 + g)
      : "memory");
  return r != 0;
}

// 4-D tensor load (activation rows: {128 B, rows, planes, K-tiles}).
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2,
                                            int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// Sum over the C accumulation chains (chain stride acc_w columns) of 16 columns
// of two column groups (the pair's blocks, half_off apart), adding the lo-plane
// columns (lo_off > 0: columns lo_off.. of the same chain); all loads of a chain
// are issued before one wait, and chains and planes are added in a fixed order,
// so the result is deterministic.
__device__ __forceinline__ void tmem_sum16x2(uint32_t taddr, uint32_t half_off, int C, uint32_t acc_w, int lo_off,
                                             float (&out0)[16], float (&out1)[16]) {
#pragma unroll
  for (int j = 0; j < 16; ++j) out0[j] = out1[j] = 0.f;
  for (int c = 0; c < C; ++c) {
    uint32_t r0[16], r1[16];
    tmem_ld16(taddr + c * acc_w, r0);
    tmem_ld16(taddr + half_off + c * acc_w, r1);
    tmem_ld_wait();
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      out0[j] += __uint_as_float(r0[j]);
      out1[j] += __uint_as_float(r1[j]);
    }
    if (lo_off) {
      tmem_ld16(taddr + c * acc_w + lo_off, r0);
      tmem_ld16(taddr + half_off + c * acc_w + lo_off, r1);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        out0[j] += __uint_as_float(r0[j]);
        out1[j] += __uint_as_float(r1[j]);
      }
    }
  }
}

// Maximum over the warp of each of 16 per-lane values by a transposed
// butterfly (16 shuffles instead of 80): lane l returns the maximum of value
// (l >> 1) & 15; both lanes of a pair hold it.
__device__ __forceinline__ float warp_colmax16(const float (&in)[16]) {
  const int lane = threadIdx.x & 31;
  float v[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = in[i];
#pragma unroll
  for (int w = 8; w >= 1; w >>= 1) {  // 16 -> 8 -> 4 -> 2 -> 1 values per lane
    const bool up = (lane & (2 * w)) != 0;
#pragma unroll
    for (int i = 0; i < w; ++i) {
      const float send = up ? v[i] : v[i + w];
      const float keep = up ? v[i + w] : v[i];
      v[i] = fmaxf(keep, __shfl_xor_sync(0xFFFFFFFFu, send, 2 * w));
    }
  }
  return fmaxf(v[0], __shfl_xor_sync(0xFFFFFFFFu, v[0], 1));
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
  // two-plane (bf16) tiles are padded to the box rows, so the lo plane sits at
  // MMA column brows + n as the activation box lays it out; E4M3 tiles to 16
  it.rpad = p.hilo ? p.brows : (it.rows + 15) & ~15;
  it.n = p.hilo ? 2 * it.rpad : it.rpad;
  return it;
}

// The ring layout is a compile-time constant of each instance (planes x token
// rows per tile), so the issuer and copier loops, unrolled over the ring, give
// every tcgen05 instruction its shared-memory and TMEM operands as immediate
// offsets from per-kernel bases.
template <int NT, int PLANES, int BROWS>
__global__ void __launch_bounds__(NT, 1)
    moe_gemm_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                    const GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int planes = PLANES;
  // E4M3 (prefill) tiles have one issuer pair, so warps 8-11 form a second
  // epilogue group: each group takes every other 16-column block of an item
  constexpr int kGroups = PLANES == 1 ? 2 : 1;
  constexpr Plan pl = make_plan(PLANES, BROWS);
  constexpr int S = pl.stages;
  static_assert(S >= 2 && S <= kMaxStages, "ring");
  uint8_t* epi = smem + pl.epi;
  Ctrl* ctrl = reinterpret_cast<Ctrl*>(epi + kEpiBytes);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const bool gu = (p.mode == 0);
  const int nbuf = p.nbuf;
  const int P = p.parities;  // stage parities split across issuer pairs (1 or 2)
  // TMEM: accumulator pair of (buffer b, chain c) at column (b*P + c) * acc_w,
  // the second block of the pair at +max_n.  Scale factors of ring stage s:
  // the pair's two weight chunks at sf_base + 12s (+4) and the token chunk at +8
  // (with the copier); without it, issuer i's weight chunk at sf_base + 8i and
  // the token chunk at +4.
  const uint32_t acc_w = static_cast<uint32_t>(2 * p.max_n);
  const uint32_t half_off = static_cast<uint32_t>(p.max_n);
  constexpr bool copier = (NT == kThreadsCopier);
  constexpr uint32_t sf_base = kTmemCols - (copier ? kSfSlotCols * static_cast<uint32_t>(S) : kSfIssuerCols);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&ctrl->full[s], 2);   // one arrival from each producer warp
      mbar_init(&ctrl->empty[s], 2 * P);  // every issuer: a commit (consumer) or an arrive (observer)
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&ctrl->acc_full[b], 2 * P);  // one commit from each issuer
      mbar_init(&ctrl->acc_empty[b], 128 * kGroups);
    }
    for (int i = 0; i < 7; ++i) mbar_init(&ctrl->drain[i], 1);
    for (int s = 0; s < S; ++s) mbar_init(&ctrl->sf_ready[s], 1);
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
  // the set-up above (barriers, TMEM, tensor-map prefetch) overlaps the previous
  // kernel's tail; everything below reads what it wrote
  griddep_wait();
  griddep_launch();

  int n_tiles = *p.n_tiles;
  if (n_tiles > p.max_tiles) n_tiles = p.max_tiles;
  const int n_items = n_tiles * p.n_blocks;
  const int KT = p.K / 128;

  // The producer, issuer and copier loops run on lane 0 alone, with the ring
  // position (stage, phase) and the accumulator position kept as counters and
  // every per-item operand computed once per item: a warp-wide loop with a
  // lane-0 branch per stage, or a division per stage, costs each
  // tcgen05.mma several hundred cycles of issue time.
  if (warp == 0 || warp == 6) {
    // ----------------------------------------------------------- producers
    if (lane == 0) {
      const bool wprod = (warp == 0);
      const uint32_t tx = wprod ? 2u * 8192u  // packed global bytes of the two weight tiles
                                : 2u * 512u + static_cast<uint32_t>(planes * p.brows) * 128u + 512u;
      int s = 0, last_s = -1;
      uint32_t ph = 0, last_ph = 0;
      bool ok = true;
      for (int item = blockIdx.x; ok && item < n_items; item += gridDim.x) {
        const Item m = get_item(p, item);
        // bank entry of the item's expert (offload: through the slot table)
        int em = m.e;
        if (p.expert_slot) {
          em = __ldg(p.expert_slot + m.e);
          if (em < 0 || em >= p.bank_slots) {
            set_error(p.err, MOSAIC_ERR_RANGE);
            em = 0;
          }
        }
        // tile index of (expert, block pair, K-tile 0, first of the pair); the two
        // tiles of the pair are adjacent for every K-tile
        const int wtile = ((em * p.n_blocks + m.nb) * KT) * 2;
        const uint8_t* sft = p.x_sft + static_cast<size_t>(m.tile) * KT * 512;
        for (int kt = 0; kt < KT; ++kt) {
          if (!mbar_wait(&ctrl->empty[s], ph ^ 1u, abort)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + s * pl.stage_bytes;
          uint64_t* fb = &ctrl->full[s];
          const int t0 = wtile + kt * 2;
          mbar_arrive_expect_tx(fb, tx);
          if (wprod) {
            tma_load_3d(st, &tmap_w, fb, 0, 0, t0);
          } else {
            tma_load_4d(st + pl.off_b, &tmap_x, fb, 0, m.row0, 0, kt);
            bulk_load(st + pl.off_sfa, p.w_sf + static_cast<size_t>(t0) * 512, 1024u, fb);
            bulk_load(st + pl.off_sfb, sft + static_cast<size_t>(kt) * 512, 512u, fb);
          }
          last_s = s;
          last_ph = ph;
          if (++s == S) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      if (!ok) {
        set_error(p.err, MOSAIC_ERR_TIMEOUT);
        ctrl->abort = 1;
      }
      // Wait (bounded) for the last armed stage so no copy is in flight at exit.
      if (last_s >= 0) {
        volatile int never = 0;
        mbar_wait(&ctrl->full[last_s], last_ph, &never);
      }
    }
    __syncwarp();
  } else if ((warp == 1 || warp >= 7) && (warp == 1 ? 0 : warp - 6) < 2 * P) {
    // ----------------------------------------------------------------- MMA
    // The whole warp runs the loop (warp-uniform operands); elect.sync inside
    // each tcgen05 instruction picks the issuing lane.
    {
      const int issuer = (warp == 1) ? 0 : warp - 6;  // 0 .. 2P-1
      const int ip = issuer >> 1;                     // stage parity this issuer takes
      const int iu = issuer & 1;                      // unit: block of the pair
      const uint32_t smem_base = smem_u32(smem);
      // descriptors of ring stage 0; stage s adds s * stage_bytes (16-byte units)
      const uint64_t ad0 = desc_sw128(smem_base + 16384u * static_cast<uint32_t>(iu));
      const uint64_t bd0 = desc_sw128(smem_base + static_cast<uint32_t>(pl.off_b));
      // scale-factor columns of ring stage 0 (copier) or of this issuer (no copier)
      const uint32_t sfw0 = copier ? tmem + sf_base + 4u * iu : tmem + sf_base + 8u * issuer;
      const uint32_t sfx0 = copier ? tmem + sf_base + 8u : tmem + sf_base + 8u * issuer + 4u;
      constexpr uint32_t sf_step = copier ? kSfSlotCols : 0u;
      int item = blockIdx.x, b = 0, kt = 0, par = 0;
      uint32_t ph = 0, aph = 0, d = 0, id0 = 0;
      bool issued = false, ok = true, live = false, done = false;
      while (!done && ok) {
#pragma unroll
        for (int s = 0; s < S; ++s) {
          if (!live) {  // next work item: its accumulator buffer must be free
            if (item >= n_items) {
              done = true;
              break;
            }
            const Item m = get_item(p, item);
            if (!mbar_wait_warp(&ctrl->acc_empty[b], aph ^ 1u, abort)) {
              ok = false;
              break;
            }
            tc_fence_after();
            d = tmem + static_cast<uint32_t>(b * P + ip) * acc_w + (iu ? half_off : 0u);
            id0 = idesc_mxf8f6f4(m.n, 0);
            kt = 0;
            par = 0;
            live = true;
          }
          // Every issuer observes every phase of every full barrier and arrives on
          // the matching empty barrier, including for the stages the other parity
          // consumes.  A parity wait that skipped phases could match the phase two
          // fills back and read a stage before it lands; requiring every issuer's
          // arrival before a refill keeps all of them within one phase of the ring.
          if (!mbar_wait_warp(copier ? &ctrl->sf_ready[s] : &ctrl->full[s], ph, abort)) {
            ok = false;
            break;
          }
          if (par != ip) {
            mbar_arrive_elect(&ctrl->empty[s]);
          } else {
            tc_fence_after();
            const uint32_t col_sfw = sfw0 + sf_step * static_cast<uint32_t>(s);
            const uint32_t col_sfx = sfx0 + sf_step * static_cast<uint32_t>(s);
            if (!copier) {
              const uint32_t sw = smem_base + static_cast<uint32_t>(s * pl.stage_bytes);
              tc_cp_32x128b_x4_elect(col_sfw, desc_sf(sw + pl.off_sfa + 512 * iu));
              tc_cp_32x128b_x4_elect(col_sfx, desc_sf(sw + pl.off_sfb));
            }
            const uint64_t so = static_cast<uint64_t>((s * pl.stage_bytes) >> 4);
            const uint32_t first = (kt < P) ? 1u : 0u;  // first stage of this issuer's chain in the item
#pragma unroll
            for (uint32_t kb = 0; kb < 4; ++kb) {
              // kb * 32 bytes along K: +2 in the descriptor's 16-byte address units
              tc_mma_mxf8f6f4_elect(d, ad0 + so + 2u * kb, bd0 + so + 2u * kb, id0 | (kb << 4) | (kb << 29),
                                    (first && kb == 0) ? 0u : 1u, col_sfw | (kb << 30), col_sfx | (kb << 30));
            }
            tc_commit_elect(&ctrl->empty[s]);
            issued = true;
          }
          if (++par == P) par = 0;
          if (++kt == KT) {  // item done: its accumulators go to the epilogue
            tc_commit_elect(&ctrl->acc_full[b]);
            issued = true;
            if (++b == nbuf) {
              b = 0;
              aph ^= 1u;
            }
            live = false;
            item += gridDim.x;
          }
        }
        ph ^= 1u;
      }
      if (!ok && lane == 0) {
        set_error(p.err, MOSAIC_ERR_TIMEOUT);
        ctrl->abort = 1;
      }
      // Drain: every MMA / copy this warp issued has completed before TMEM is freed.
      if (issued) {
        tc_commit_elect(&ctrl->drain[issuer]);
        volatile int never = 0;
        mbar_wait_warp(&ctrl->drain[issuer], 0, &never);
      }
    }
    __syncwarp();
  } else if (warp == 12 && copier) {
    // -------------------------------------------------- scale-factor copier
    {
      const uint32_t smem_base = smem_u32(smem);
      const uint64_t sd0 = desc_sf(smem_base + static_cast<uint32_t>(pl.off_sfa));
      const uint64_t xd0 = desc_sf(smem_base + static_cast<uint32_t>(pl.off_sfb));
      int item = blockIdx.x, kt = 0;
      uint32_t ph = 0;
      bool issued = false, ok = true, done = item >= n_items;
      while (!done && ok) {
#pragma unroll
        for (int s = 0; s < S; ++s) {
          if (!mbar_wait_warp(&ctrl->full[s], ph, abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t so = static_cast<uint64_t>((s * pl.stage_bytes) >> 4);
          const uint32_t c0 = tmem + sf_base + kSfSlotCols * static_cast<uint32_t>(s);
          tc_cp_32x128b_x4_elect(c0, sd0 + so);
          tc_cp_32x128b_x4_elect(c0 + 4u, sd0 + so + 32u);  // + 512 bytes
          tc_cp_32x128b_x4_elect(c0 + 8u, xd0 + so);
          tc_commit_elect(&ctrl->sf_ready[s]);
          issued = true;
          if (++kt == KT) {
            kt = 0;
            item += gridDim.x;
            if (item >= n_items) {
              done = true;
              break;
            }
          }
        }
        ph ^= 1u;
      }
      if (!ok && lane == 0) {
        set_error(p.err, MOSAIC_ERR_TIMEOUT);
        ctrl->abort = 1;
      }
      if (issued) {
        tc_commit_elect(&ctrl->drain[6]);
        volatile int never = 0;
        mbar_wait_warp(&ctrl->drain[6], 0, &never);
      }
    }
    __syncwarp();
  } else if ((warp >= 2 && warp <= 5) || (kGroups == 2 && warp >= 8 && warp <= 11)) {
    // ------------------------------------------------------------ epilogue
    // Warp w reads TMEM lanes 32*(w%4).. (weight rows); each thread holds one
    // weight row of 16 token columns at a time.  Per item, the rows' route
    // weights (gate/up) or output rows (down) are loaded into shared memory
    // once; per 16-column block, column maxima use transposed butterflies and
    // the staging buffers alternate between blocks, so a gate/up block takes
    // two named barriers.  With two groups (warps 2-5 and 8-11), group g takes
    // the blocks starting at columns 16g, 16g + 32, ... with its own barrier,
    // metadata and half of the staging area.
    const int g = warp >= 8 ? 1 : 0;
    const int q = warp & 3;
    const int lrow = q * 32 + lane;
    const int et = (warp - (g ? 8 : 2)) * 32 + lane;  // 0..127: this thread's index in its group
    const uint32_t tq = tmem + (static_cast<uint32_t>(q * 32) << 16);
    const size_t z_plane = static_cast<size_t>(p.R_pad) * 128;    // bytes per (K-tile, plane) of z rows
    const size_t z_ktile = static_cast<size_t>(planes) * z_plane;  // bytes per K-tile of z rows
    uint8_t* epi_g = epi + g * (kEpiBytes / kGroups);
    float* stage_f = reinterpret_cast<float*>(epi_g);              // down, fp32: [16 tokens][256 values]
    __nv_bfloat16* stage_h = reinterpret_cast<__nv_bfloat16*>(epi_g);  // down, bf16: [16 tokens][256 values]
    float* meta_w = ctrl->meta_w[g];
    int* meta_o = ctrl->meta_o[g];
    int* meta_r = ctrl->meta_r[g];
    const int P_used = KT < P ? KT : P;                            // chains that received MMAs
    int li = 0, blk = 0;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x, ++li) {
      const Item m = get_item(p, item);
      const bool round_mid = p.fp8 || (m.e == p.shared_expert);
      const int b = li % nbuf;
      const uint32_t aph = static_cast<uint32_t>(li / nbuf) & 1u;
      // row metadata of the item (read by every warp after the barrier below)
      if (et < m.rows) {
        const int r = m.row0 + et;
        if (gu) {
          meta_w[et] = p.row_weight[r];
        } else if (p.ep_row_pos) {  // unit rows: the return rank and row of packed row r
          meta_r[et] = p.ep_row_rank[r];
          meta_o[et] = p.ep_row_pos[r];
        } else {
          const int orow = p.out_row ? p.out_row[r] : r;
          if (p.ep_world) {  // receive row orow of source s goes to s's send position of it
            int sr = 0;
            while (sr + 1 < p.ep_world && orow >= p.ep_recv_start[sr + 1]) ++sr;
            meta_r[et] = sr;
            meta_o[et] = p.ep_src_pos[sr] + orow - p.ep_recv_start[sr];
          } else {
            meta_o[et] = orow;
          }
        }
      }
      // every epilogue warp takes the same branch (a warp that left while the
      // others wait at a named barrier would hold them there)
      if (!epi_all(g, mbar_wait_warp(&ctrl->acc_full[b], aph, abort))) {  // also makes the metadata visible
        if (lane == 0) {
          set_error(p.err, MOSAIC_ERR_TIMEOUT);
          ctrl->abort = 1;
        }
        break;
      }
      tc_fence_after();
      const uint32_t c_buf = static_cast<uint32_t>(b * P) * acc_w;
      const int lo = p.hilo ? m.rpad : 0;
      for (int c0 = 16 * g; c0 < m.rpad; c0 += 16 * kGroups, ++blk) {
        float s0[16], s1[16];
        tmem_sum16x2(tq + c_buf + c0, half_off, P_used, acc_w, lo, s0, s1);
        const int ncol = min(16, m.rows - c0);  // token columns of this block that exist
        if (gu) {
          uint8_t* stage_b = epi_g + (blk & 1) * 4096;  // [planes][16 tokens][128 B], alternating
          float4* red = ctrl->red4[g][blk & 1];
          float zd[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            float gv = s0[j];
            float uv = s1[j];
            if (round_mid) {
              gv = bf16r(gv);
              uv = bf16r(uv);
            }
            if (p.swiglu_limit > 0.f) {
              gv = fminf(gv, p.swiglu_limit);
              uv = fminf(fmaxf(uv, -p.swiglu_limit), p.swiglu_limit);
            }
            const float w = (j < ncol) ? meta_w[c0 + j] : 0.f;
            float z = gv / (1.0f + expf(-gv)) * uv;
            z = z * w;
            zd[j] = (j < ncol) ? bf16r(z) : 0.f;
          }
          // quantised bytes staged as [plane][token][128 B] (this thread: byte lrow)
          uint32_t* zsf = p.z_sft + (static_cast<size_t>(m.tile) * (p.I / 128) + m.nb) * 128;
          if (p.fp8) {
            // act_quant per 128 rows: column maxima of the four warps meet in shared memory
            float a[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) a[j] = fabsf(zd[j]);
            const float cm = warp_colmax16(a);
            if ((lane & 1) == 0) reinterpret_cast<float*>(&red[(lane >> 1) & 15])[q] = cm;
            epi_bar(g);
            int my_ex = 0;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const float4 r4 = red[j];
              const float amax = fmaxf(fmaxf(r4.x, r4.y), fmaxf(r4.z, r4.w));
              const int ex = pow2_scale_exp(amax, 1e-4f);
              if (j == lrow) my_ex = ex;
              const float y = fminf(fmaxf(zd[j] * exp2i(-ex), -448.f), 448.f);
              stage_b[j * 128 + lrow] = f32_to_e4m3(y);
            }
            if (lrow < ncol) zsf[sf_word(c0 + lrow)] = (static_cast<uint32_t>(my_ex + 127) & 0xFFu) * 0x01010101u;
          } else {
            // hi + lo planes with per-32-row (per-warp) scales
            float a[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) a[j] = fabsf(zd[j]);
            const float cm = warp_colmax16(a);
            float res[16];
            int eh[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const float mx = __shfl_sync(0xFFFFFFFFu, cm, 2 * j);
              eh[j] = max(-126, min(127, pow2_scale_exp(mx, 1e-30f)));
              const uint8_t hb = f32_to_e4m3(zd[j] * exp2i(-eh[j]));
              res[j] = zd[j] - e4m3_to_f32(hb) * exp2i(eh[j]);
              stage_b[j * 128 + lrow] = hb;
              a[j] = fabsf(res[j]);
              s0[j] = mx;  // keep the hi maximum for the lo floor
            }
            const float cm2 = warp_colmax16(a);
            int my_e = 0;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const float m2 = __shfl_sync(0xFFFFFFFFu, cm2, 2 * j);
              const int el = max(-126, min(127, pow2_scale_exp(m2, fmaxf(s0[j] * 1e-7f, 1e-30f))));
              stage_b[2048 + j * 128 + lrow] = f32_to_e4m3(res[j] * exp2i(-el));
              if ((lane & 15) == j) my_e = (lane < 16) ? eh[j] : el;
            }
            // lane j writes the hi exponent of column j, lane 16 + j the lo one
            const int jc = lane & 15;
            if (jc < ncol) {
              const int col = (lane < 16) ? c0 + jc : m.rpad + c0 + jc;
              reinterpret_cast<uint8_t*>(zsf + sf_word(col))[q] = static_cast<uint8_t>(my_e + 127);
            }
          }
          epi_bar(g);
          // 16-byte stores of whole 128-byte z rows: planes x 16 tokens x 8 vectors
          uint8_t* zq = p.zq + static_cast<size_t>(m.nb) * z_ktile;
          for (int v = et; v < planes * 128; v += 128) {
            const int pl_ = v >> 7, j = (v >> 3) & 15, off = (v & 7) * 16;
            if (j < ncol)
              *reinterpret_cast<uint4*>(zq + pl_ * z_plane + static_cast<size_t>(m.row0 + c0 + j) * 128 + off) =
                  *reinterpret_cast<const uint4*>(stage_b + pl_ * 2048 + j * 128 + off);
          }
          // the next block writes the other staging buffer and the other maxima
        } else {
          // partials of the two hidden blocks, staged as [token][256 values]
          // (fp32 partials as fp32, bf16 ones rounded here)
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            float v0 = s0[j], v1 = s1[j];
            if (round_mid) {
              v0 = bf16r(v0);
              v1 = bf16r(v1);
            }
            if (p.out_f32) {
              stage_f[j * 256 + lrow] = v0;
              stage_f[j * 256 + 128 + lrow] = v1;
            } else {
              stage_h[j * 256 + lrow] = __float2bfloat16_rn(v0);
              stage_h[j * 256 + 128 + lrow] = __float2bfloat16_rn(v1);
            }
          }
          epi_bar(g);
          // 16-byte stores: per token, two runs of 128 values (block nb of each half)
          const int hb = p.H / 2;
          const int esz = p.out_f32 ? 4 : 2;
          const int per = p.out_f32 ? 32 : 16;  // 16-byte vectors per run of 128 values
          for (int v = et; v < 16 * 2 * per; v += 128) {
            const int j = v / (2 * per), h = (v / per) & 1, w16 = v % per;
            if (j >= ncol) continue;
            const int orow = meta_o[c0 + j];
            uint8_t* row_base = p.ep_world ? p.ep_regions[meta_r[c0 + j]] + p.ep_ret_off +
                                                 static_cast<size_t>(orow) * p.H * esz
                                           : static_cast<uint8_t*>(p.out) + static_cast<size_t>(orow) * p.H * esz;
            uint4* dst = reinterpret_cast<uint4*>(row_base + static_cast<size_t>(h * hb + m.nb * 128) * esz) + w16;
            *dst = p.out_f32 ? reinterpret_cast<const uint4*>(stage_f + j * 256 + h * 128)[w16]
                             : reinterpret_cast<const uint4*>(stage_h + j * 256 + h * 128)[w16];
          }
          epi_bar(g);
        }
      }
      tc_fence_before();
      mbar_arrive(&ctrl->acc_empty[b]);
      epi_bar(g);  // every warp is done with this item's metadata before the next item's is written
    }
    // partials stored into other ranks' memory are made visible at system
    // scope before the kernel ends (the next kernel stamps their flags)
    if (p.ep_world) __threadfence_system();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

}  // namespace

size_t gemm_smem_bytes(int planes, int brows) {
  const Plan pl = make_plan(planes, brows);
  return static_cast<size_t>(pl.stages) * pl.stage_bytes + kEpiBytes + sizeof(Ctrl) + 1024;
}

cudaError_t launch_moe_gemm(const CUtensorMap& tmap_w, const CUtensorMap& tmap_x, const GemmParams& p, int grid,
                            cudaStream_t stream) {
  if (p.max_n < 16 || p.max_n > 128 || p.nbuf < 1 || p.nbuf > 2 || p.parities < 1 || p.parities > kMaxParities)
    return cudaErrorInvalidValue;
  const int planes = p.hilo ? 2 : 1;
  if (p.brows * planes != p.max_n || p.brows % 16 || p.brows > 128) return cudaErrorInvalidValue;
  {
    const Plan pl0 = make_plan(p.hilo ? 2 : 1, p.brows);
    const int sf_cols = p.sf_copier ? static_cast<int>(kSfSlotCols) * pl0.stages : static_cast<int>(kSfIssuerCols);
    if (p.nbuf * p.parities * 2 * p.max_n > static_cast<int>(kTmemCols) - sf_cols)
      return cudaErrorInvalidValue;
  }
  if (p.K % 128 || p.K < 128) return cudaErrorInvalidValue;
  if (p.mode == 1 && p.H % 256) return cudaErrorInvalidValue;
  // the E4M3 instance runs two epilogue groups on the warps of the unused issuer
  // pairs, each staging bf16 partials in half of the staging area
  if (!p.hilo && (p.parities != 1 || (p.mode == 1 && p.out_f32))) return cudaErrorInvalidValue;
  const Plan pl = make_plan(planes, p.brows);
  if (pl.stages < 2) return cudaErrorInvalidValue;
  const size_t smem = gemm_smem_bytes(planes, p.brows);
  // the three tile shapes the workspace plans use: E4M3 tiles of 112 rows
  // (double-buffered, no copier: the issuers' own scale copies beat the copier's
  // extra barrier hop per stage there), two-plane tiles of 16 rows
  // (double-buffered, with the copier) and of 32 rows (single-buffered, no copier)
  void (*kernel)(const CUtensorMap, const CUtensorMap, const GemmParams) = nullptr;
  if (planes == 1 && p.brows == 112 && !p.sf_copier) kernel = moe_gemm_kernel<kThreadsPlain, 1, 112>;
  if (planes == 2 && p.brows == 16 && p.sf_copier) kernel = moe_gemm_kernel<kThreadsCopier, 2, 16>;
  if (planes == 2 && p.brows == 32 && !p.sf_copier) kernel = moe_gemm_kernel<kThreadsPlain, 2, 32>;
  if (!kernel) return cudaErrorInvalidValue;
  cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
  if (err != cudaSuccess) return err;
  err = launch_k(kernel, dim3(grid), dim3(p.sf_copier ? kThreadsCopier : kThreadsPlain), smem, stream, tmap_w, tmap_x,
                 p);
  if (err != cudaSuccess) return err;
  return cudaGetLastError();
}

}  // namespace mosaic
