// Grouped expert GEMMs on the 5th-generation tensor cores (tcgen05 + TMEM),
// fed by TMA. One persistent kernel template serves both matmuls of the MoE
// layer (kernels/track1-triton/fused_moe/base.py:69-72):
//
//   gate-up: act[m, :] = silu(A[m] . W13g[e]^T) * (A[m] . W13u[e]^T)
//            (base.py:69-71; the SiLU(gate)*up epilogue is fused)
//   down:    part[s, r, :] = w[r] * (act[m] . W2[e]^T)   restricted to K split s
//            (base.py:72 and the topk-weight multiply of base.py:75)
//
// where m runs over the rows of the expert-sorted operand, r = sorted_ids[m]
// is the flat (token, slot) index and e = expert_ids[m / 128].
//
// CTA layout (320 threads, one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: A tile [128 x 128 B] + B tile [BN x 128 B] per
//               k-block into a STAGES-deep shared-memory ring.
//   warp 1      allocates 2*BN TMEM columns; lane 0 issues tcgen05.mma
//               (M=128, N=BN, 4 MMAs per 128-byte k-block) into one of two
//               accumulator buffers, so the epilogue of tile i overlaps the
//               main loop of tile i+1.
//   warps 2..9  epilogue: warp w reads TMEM lane quarter w % 4 and column
//               half (w - 2) / 4, several 32-lane x 16-column tcgen05.ld per
//               wait, fused math, 16-byte stores to global memory.
// Tiles are (m-block, n-tile, k-split) triples handed out round-robin, group
// by group: a group is one expert's run of m-blocks (at most kGroupMax; a
// longer run is split evenly) and inside it the n-tile index varies slowest,
// so the CTAs running at the same time share each weight tile through L2
// and an expert's weights stream from DRAM once per group.
//
// Launched with programmatic dependent launch: given early metadata (the
// align outputs are two launches old), the producer requests the weight
// tiles of its first stages before waiting on the kernel that wrote A.
//
// The fp8 block-scaled variant (moe_grouped_gemm_fp8_kernel, below) uses 20
// warps: a per-k-block TMEM buffer is promoted into fp32 registers by 16
// epilogue warps with the activation and weight block scales. With
// power-of-two (UE8M0) scales the tensor core applies them itself
// (moe_grouped_gemm_mx_kernel, kind::mxf8f6f4.block_scale) and the tile
// accumulates in TMEM like the bf16 kernel's.
//
// Every barrier wait is bounded (one second): a role that runs out raises a
// shared abort flag, every role leaves its loop, in-flight TMA loads and
// MMAs are waited for, TMEM is freed and MOE_ERR_TIMEOUT is reported.
#include <atomic>
#include <cstdlib>
#include <type_traits>

#include "common.cuh"
#include "internal.h"
#include "runtime.h"

namespace ksw {
namespace {

constexpr int BM = kBlockM;          // rows per tile (TMEM lanes)
constexpr int kKBytes = 128;         // bytes of K per k-block (one swizzle row)
constexpr int kABytes = BM * kKBytes;
constexpr int kThreads = 320;  // producer, MMA, 8 epilogue warps
constexpr int kGroupM = 8;

enum Epi : int { kEpiSwiGLU = 0, kEpiRows = 1 };

struct KParams {
  const int32_t* num_post_pad;
  const int32_t* expert_ids;
  const int32_t* sorted_ids;
  const float* a_scale;     // INT8: [rows]; FP8_UE8M0: scale-factor image (bytes)
  const float* b_scale;     // INT8: [E, n]; FP8_UE8M0: scale-factor image (bytes)
  const void* row_weights;  // down: [numel]
  void* out;
  int32_t* status;
  int64_t out_ld;           // elements between output rows
  int32_t max_m_blocks;
  int32_t n_total;
  int32_t k_blocks;
  int32_t splits;
  int32_t kb_per_split;
  int32_t numel;
  int32_t num_experts;
  int32_t row_weights_dtype;
  // FP8 block scales: a_scale [rows, sa_ld], b_scale [E, sb_rb, sb_kb]
  int32_t sa_ld;
  int32_t sb_rb;
  int32_t sb_kb;
  int32_t up_offset;        // gate-up: original row of the first up row (= I)
  int32_t early_meta;       // see GroupedGemmArgs::early_meta
  int32_t tail_halves;      // 256-wide unsplit rows epilogue: see moe_grouped_gemm_kernel
  uint64_t wait_limit_ns;
};

struct TileCoord {
  int mb, nt, ks;
  int half;  // -1: the whole BN-wide tile; 0 / 1: its first / second 128 columns
};

// ---------------------------------------------------------------------------
// Expert-aligned tile groups. Tiles are enumerated group by group; inside a
// group of m-blocks the n-tile varies slowest, so the CTAs that run the
// group's m-blocks at the same time share each weight tile through L2.
// Groups follow the experts: a run of m-blocks of one expert forms one group
// (split into near-equal chunks of at most kGroupMax m-blocks), so an
// expert's weights are streamed once per chunk instead of once more for
// every fixed-size group boundary that falls inside the run. Entry m of the
// table: (first m-block of m's group) << 16 | (the group's m-blocks).
// ---------------------------------------------------------------------------
constexpr int kGroupMax = 16;
constexpr int kMaxTableMb = 4096;  // larger problems use the fixed groups below
constexpr size_t kGroupTableBytes = size_t(kMaxTableMb) * 4 + 256;

// Block-wide inclusive scan of v (max, or min when MIN) in thread order;
// `carry` joins consecutive calls. All threads call it; scratch >= 33 ints.
template <bool MIN>
__device__ __forceinline__ int block_scan(int v, int& carry, int* scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  auto op = [](int x, int y) { return MIN ? min(x, y) : max(x, y); };
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v = op(v, y);
  }
  if (lane == 31) scratch[warp] = v;
  __syncthreads();
  if (warp == 0) {
    int w = lane < nw ? scratch[lane] : (MIN ? INT_MAX : INT_MIN);
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w = op(w, y);
    }
    scratch[lane] = w;
  }
  __syncthreads();
  if (warp > 0) v = op(v, scratch[warp - 1]);
  v = op(v, carry);
  const int total = op(scratch[nw - 1], carry);
  __syncthreads();
  carry = total;
  return v;
}

// Builds the group table for m-blocks [0, num_mb) (num_mb <= kMaxTableMb).
// All threads of the block call it.
__device__ void build_group_table(const int32_t* __restrict__ expert_ids, int num_mb,
                                  uint32_t* tab, int* scratch) {
  const int nthr = blockDim.x;
  // pass 1: tab[m] = first m-block of m's run (max-scan of run starts)
  int carry = 0;
  for (int base = 0; base < num_mb; base += nthr) {
    const int m = base + threadIdx.x;
    int v = 0;
    if (m < num_mb && (m == 0 || __ldg(expert_ids + m) != __ldg(expert_ids + m - 1))) v = m;
    v = block_scan<false>(v, carry, scratch);
    if (m < num_mb) tab[m] = uint32_t(v);
  }
  __syncthreads();
  // pass 2: run end = the next run start after m (min-scan from the right);
  // tab[m] = start | end << 16 (the low half, read by the neighbours, stays)
  carry = num_mb;
  for (int base = ((num_mb - 1) / nthr) * nthr; base >= 0; base -= nthr) {
    const int m = base + (nthr - 1 - threadIdx.x);  // descending in thread order
    int v = num_mb;
    if (m + 1 < num_mb && m >= 0 && int(tab[m + 1] & 0xFFFFu) == m + 1) v = m + 1;
    v = block_scan<true>(v, carry, scratch);
    if (m >= 0 && m < num_mb) tab[m] = (tab[m] & 0xFFFFu) | (uint32_t(v) << 16);
    __syncthreads();
  }
  // pass 3: chunk the run, store (group start, group size)
  for (int m = threadIdx.x; m < num_mb; m += nthr) {
    const int start = int(tab[m] & 0xFFFFu), end = int(tab[m] >> 16);
    const int len = end - start;
    const int chunks = (len + kGroupMax - 1) / kGroupMax;
    const int csz = (len + chunks - 1) / chunks;
    const int gs = start + ((m - start) / csz) * csz;
    tab[m] = (uint32_t(gs) << 16) | uint32_t(min(csz, end - gs));
  }
  __syncthreads();
}

__device__ __forceinline__ TileCoord tile_coord_tab(int t, int n_tiles, int splits,
                                                    const uint32_t* tab) {
  TileCoord c;
  c.half = -1;
  c.ks = t % splits;
  const int u = t / splits;
  const uint32_t e = tab[u / n_tiles];
  const int gs = int(e >> 16), gsz = int(e & 0xFFFFu);
  const int v = u - gs * n_tiles;
  c.nt = v / gsz;
  c.mb = gs + (v - c.nt * gsz);
  return c;
}

__device__ __forceinline__ TileCoord tile_coord(int t, int num_mb, int n_tiles,
                                                int splits) {
  TileCoord c;
  c.half = -1;
  c.ks = t % splits;
  const int u = t / splits;
  const int per_group = kGroupM * n_tiles;
  const int g = u / per_group;
  const int v = u - g * per_group;
  const int gm = min(kGroupM, num_mb - g * kGroupM);
  c.nt = v / gm;
  c.mb = g * kGroupM + (v - c.nt * gm);
  return c;
}

__device__ __forceinline__ float silu_mul(float g, float u) {
  return g / (1.0f + __expf(-g)) * u;
}

// Weight of flat row i; a null weight array means unit weights (the
// unweighted partial rows of the split-K gate-up GEMM).
__device__ __forceinline__ float load_weight(const void* w, int dtype,
                                             int64_t i) {
  if (w == nullptr) return 1.0f;
  if (dtype == MOE_DTYPE_F32) return static_cast<const float*>(w)[i];
  if (dtype == MOE_DTYPE_BF16)
    return __bfloat162float(static_cast<const __nv_bfloat16*>(w)[i]);
  return __half2float(static_cast<const __half*>(w)[i]);
}

template <int KIND>
__device__ __forceinline__ float acc_to_f32(uint32_t v) {
  if constexpr (KIND == kKindI8)
    return static_cast<float>(static_cast<int32_t>(v));
  else
    return __uint_as_float(v);
}

template <int BN>
struct GemmCfg {
  static constexpr int kBBytes = BN * kKBytes;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = (192 * 1024) / kStageBytes;
  static constexpr int kTmemCols = 2 * BN;
  static constexpr size_t kSmemBytes =
      1024 + size_t(kStages) * kStageBytes + 256 + kGroupTableBytes;
  static_assert(kStages >= 2, "pipeline needs at least two stages");
  static_assert(kTmemCols >= 32 && kTmemCols <= 512, "TMEM columns");
};

// KIND: kKindF16 (AB_FMT 0 = f16, 1 = bf16), kKindTF32 (AB_FMT 2, fp32
// operands read as tf32) or kKindI8 (AB_FMT 1 = s8).
// TOUT: element type of the gate-up output (f16/bf16).
//
// Tail halves (rows epilogue, BN = 256, no K split, p.tail_halves): when the
// tiles do not fill the last wave of CTAs and the remainder R is at most half
// the grid, those R tiles run as 2R items of 128 columns each (tmB128 loads
// 128 weight rows, the MMA runs N = 128, the epilogue covers the item's
// columns), so the last wave takes about half a tile-time instead of a full
// one. Each output element keeps its K order: results are unchanged.
template <int KIND, int AB_FMT, int BN, int EPI, typename TOUT>
__global__ void __launch_bounds__(kThreads, 1)
    moe_grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmA,
                            const __grid_constant__ CUtensorMap tmB,
                            const __grid_constant__ CUtensorMap tmB128,
                            const KParams p) {
  using Cfg = GemmCfg<BN>;
  constexpr int STAGES = Cfg::kStages;
  constexpr uint32_t D_FMT = (KIND == kKindI8) ? 2u : 1u;
  constexpr uint32_t IDESC = make_idesc(D_FMT, AB_FMT, BM, BN);
  constexpr uint32_t IDESC_HALF = make_idesc(D_FMT, AB_FMT, BM, 128);
  constexpr bool kHalves = (EPI == kEpiRows && BN == 256);
  constexpr bool kScaled = (KIND == kKindI8);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + STAGES * kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * Cfg::kBBytes);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* final_bar = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(final_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  static_assert(8 * (2 * STAGES + 5) + 8 <= 256, "barrier area");

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 256);
    }
    mbar_init(final_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // Programmatic dependent launch: without early metadata every thread
  // waits for the previous kernel here; with it, the align outputs are read
  // first (they were written two launches earlier), and only the A loads
  // (and so everything downstream of them) wait, after the first weight
  // tiles have been requested.
  const bool producer = warp == 0 && lane == 0;
  const bool early = p.early_meta;
  if (!early) {
    pdl_wait();
    pdl_trigger();
  }
  const int num_mb = min(__ldg(p.num_post_pad) / BM, p.max_m_blocks);
  const int n_tiles = p.n_total / BN;
  const int total_tiles = num_mb * n_tiles * p.splits;
  const uint64_t limit = p.wait_limit_ns;
  uint32_t* gtab = reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(full) + 256);
  const bool use_tab = num_mb <= kMaxTableMb;
  if (use_tab)
    build_group_table(p.expert_ids, num_mb, gtab, reinterpret_cast<int*>(gtab + kMaxTableMb));
  auto coord = [&](int t) {
    return use_tab ? tile_coord_tab(t, n_tiles, p.splits, gtab)
                   : tile_coord(t, num_mb, n_tiles, p.splits);
  };
  // item i -> its coordinates and k-block range (tail halves: items past
  // full_tiles are the 128-column halves of the remaining tiles)
  int full_tiles = total_tiles;
  if constexpr (kHalves) {
    const int rem = total_tiles % int(gridDim.x);
    if (p.tail_halves && p.splits == 1 && rem != 0 && 2 * rem <= int(gridDim.x))
      full_tiles = total_tiles - rem;
  }
  const int total_items = full_tiles + 2 * (total_tiles - full_tiles);
  auto item = [&](int i, TileCoord& c, int& kb0, int& kb1) {
    if (i < full_tiles) {
      c = coord(i);
    } else {
      const int hi = i - full_tiles;
      c = coord(full_tiles + (hi >> 1));
      c.half = hi & 1;
    }
    kb0 = c.ks * p.kb_per_split;
    kb1 = min(kb0 + p.kb_per_split, p.k_blocks);
  };
  // weight rows, tensor map and transaction bytes of an item's stages
  auto b_first_row = [&](int e, const TileCoord& c) {
    return e * p.n_total + c.nt * BN + (c.half > 0 ? 128 : 0);
  };
  auto b_map = [&](const TileCoord& c) { return c.half >= 0 ? &tmB128 : &tmB; };
  auto stage_bytes = [&](const TileCoord& c) {
    return uint32_t(c.half >= 0 ? kABytes + 128 * kKBytes : Cfg::kStageBytes);
  };
  if (early && !producer) {
    pdl_wait();
    pdl_trigger();
  }

  if (producer) {
    // ---------------- TMA producer ----------------
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    constexpr int kColsPerKb = kKBytes / (KIND == kKindF16 ? 2 : KIND == kKindTF32 ? 4 : 1);
    // With early metadata the weight tiles of the first STAGES k-blocks (in
    // the order the main loop visits them) are requested before the wait
    // for the A operand's producer; those stages later get only their A tile.
    uint32_t pre = 0;
    if (p.early_meta) {
      for (int t = blockIdx.x; pre < uint32_t(STAGES) && t < total_items; t += gridDim.x) {
        TileCoord c;
        int kb0, kb1;
        item(t, c, kb0, kb1);
        const int e = __ldg(p.expert_ids + c.mb);
        if (e < 0 || e >= p.num_experts) continue;
        const int b_row = b_first_row(e, c);
        for (int kb = kb0; kb < kb1 && pre < uint32_t(STAGES); ++kb, ++pre) {
          mbar_arrive_expect_tx(&full[pre], stage_bytes(c));
          tma_load_2d(sB + pre * Cfg::kBBytes, b_map(c), kb * kColsPerKb, b_row, &full[pre]);
        }
      }
      pdl_wait();
      pdl_trigger();
    }
    int stage = 0;
    uint32_t phase = 0;
    uint32_t issued = 0;
    bool ok = true;
    for (int t = blockIdx.x; ok && t < total_items; t += gridDim.x) {
      TileCoord c;
      int kb0, kb1;
      item(t, c, kb0, kb1);
      const int e = __ldg(p.expert_ids + c.mb);
      if (e < 0 || e >= p.num_experts) continue;
      const int a_row = c.mb * BM;
      const int b_row = b_first_row(e, c);
      for (int kb = kb0; kb < kb1; ++kb) {
        const int kcol = kb * kColsPerKb;
        if (issued < pre) {
          // first pass over the ring (stage == issued): B is on its way
          tma_load_2d(sA + stage * kABytes, &tmA, kcol, a_row, &full[stage]);
        } else {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1u, abort_flag, limit)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], stage_bytes(c));
          tma_load_2d(sA + stage * kABytes, &tmA, kcol, a_row, &full[stage]);
          tma_load_2d(sB + stage * Cfg::kBBytes, b_map(c), kcol, b_row, &full[stage]);
        }
        ++issued;
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    // Drain: every load issued into a stage must have landed before the CTA
    // may exit (on the normal path they have all been consumed already).
    for (int s = 0; s < STAGES; ++s) {
      const uint32_t n_s = issued / STAGES + (uint32_t(s) < issued % STAGES ? 1u : 0u);
      if (n_s == 0) continue;
      volatile int no_abort = 0;
      mbar_wait_bounded(&full[s], (n_s - 1) & 1u, &no_abort, limit);
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer ----------------
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    for (int t = blockIdx.x; ok && t < total_items; t += gridDim.x) {
      TileCoord c;
      int kb0, kb1;
      item(t, c, kb0, kb1);
      const int e = __ldg(p.expert_ids + c.mb);
      if (e < 0 || e >= p.num_experts) continue;
      if (!mbar_wait_bounded(&tempty[acc], acc_phase ^ 1u, abort_flag, limit)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + uint32_t(acc * BN);
      const uint32_t idesc = c.half >= 0 ? IDESC_HALF : IDESC;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait_bounded(&full[stage], phase, abort_flag, limit)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a0 = smem_u32(sA + stage * kABytes);
        const uint32_t b0 = smem_u32(sB + stage * Cfg::kBBytes);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          tc_mma<KIND>(d_tmem, make_sw128_desc(a0 + kk * 32),
                       make_sw128_desc(b0 + kk * 32), idesc,
                       (kb > kb0 || kk > 0) ? 1u : 0u);
        }
        tc_commit(&empty[stage]);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) break;
      tc_commit(&tfull[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
    // All MMAs issued by this thread must complete before TMEM is freed.
    tc_commit(final_bar);
    volatile int no_abort = 0;
    mbar_wait_bounded(final_bar, 0, &no_abort, limit);
  } else if (warp >= 2) {
    // ---------------- epilogue (8 warps) ----------------
    // warp w (2..9) reads TMEM lane quarter w % 4 and column half (w - 2) / 4
    const int q = warp & 3;
    const int h = (warp - 2) >> 2;
    const int row = q * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < total_items; t += gridDim.x) {
      TileCoord c;
      int kb0, kb1;
      item(t, c, kb0, kb1);
      const int e = __ldg(p.expert_ids + c.mb);
      if (e < 0 || e >= p.num_experts) continue;
      bool ok = mbar_wait_bounded(&tfull[acc], acc_phase, abort_flag, limit);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      const int m = c.mb * BM + row;
      const int r = __ldg(p.sorted_ids + m);
      const bool valid = r < p.numel;
      const uint32_t tbase =
          tmem_base + (uint32_t(q * 32) << 16) + uint32_t(acc * BN);
      float a_s = 1.0f;
      if constexpr (kScaled) a_s = valid ? __ldg(p.a_scale + m) : 0.0f;
      const int col0 = c.nt * BN + (c.half > 0 ? 128 : 0);  // the item's first column
      const float* bsc = kScaled ? p.b_scale + int64_t(e) * p.n_total + col0 : nullptr;

      if constexpr (EPI == kEpiSwiGLU) {
        constexpr int G_HALF = BN / 64;              // 32-column groups per half
        constexpr int GPI = G_HALF >= 2 ? 2 : 1;     // groups per TMEM wait
        TOUT* out_row = static_cast<TOUT*>(p.out) + int64_t(m) * p.out_ld +
                        c.nt * (BN / 2);
#pragma unroll 1
        for (int gg = 0; gg < G_HALF; gg += GPI) {
          uint32_t gv[GPI][16], uv[GPI][16];
#pragma unroll
          for (int u = 0; u < GPI; ++u) {
            const int g = h * G_HALF + gg + u;
            tmem_ld16(tbase + g * 32, gv[u]);
            tmem_ld16(tbase + g * 32 + 16, uv[u]);
          }
          tmem_ld_wait();
          if (valid) {
#pragma unroll
            for (int u = 0; u < GPI; ++u) {
              const int g = h * G_HALF + gg + u;
              float gs[16], us[16];
              if constexpr (kScaled) {
                // per-column weight scales of this 32-column group, times the row scale
                const float4* sg = reinterpret_cast<const float4*>(bsc + g * 32);
#pragma unroll
                for (int q4 = 0; q4 < 4; ++q4) {
                  const float4 a4 = __ldg(sg + q4), b4 = __ldg(sg + 4 + q4);
                  gs[4 * q4] = a_s * a4.x; gs[4 * q4 + 1] = a_s * a4.y;
                  gs[4 * q4 + 2] = a_s * a4.z; gs[4 * q4 + 3] = a_s * a4.w;
                  us[4 * q4] = a_s * b4.x; us[4 * q4 + 1] = a_s * b4.y;
                  us[4 * q4 + 2] = a_s * b4.z; us[4 * q4 + 3] = a_s * b4.w;
                }
              }
              if constexpr (std::is_same<TOUT, float>::value) {
                // fp32 activations (the down GEMM's tf32 operand, rounded
                // to tf32 here): 16 floats per group
                float4* dst = reinterpret_cast<float4*>(out_row + g * 16);
                auto act_at = [&](int j) {
                  return round_tf32(silu_mul(acc_to_f32<KIND>(gv[u][j]),
                                             acc_to_f32<KIND>(uv[u][j])));
                };
#pragma unroll
                for (int j = 0; j < 4; ++j)
                  dst[j] = make_float4(act_at(4 * j), act_at(4 * j + 1), act_at(4 * j + 2),
                                       act_at(4 * j + 3));
              } else {
                uint32_t packed[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                  float g0 = acc_to_f32<KIND>(gv[u][2 * j]);
                  float g1 = acc_to_f32<KIND>(gv[u][2 * j + 1]);
                  float u0 = acc_to_f32<KIND>(uv[u][2 * j]);
                  float u1 = acc_to_f32<KIND>(uv[u][2 * j + 1]);
                  if constexpr (kScaled) {
                    g0 *= gs[2 * j];
                    g1 *= gs[2 * j + 1];
                    u0 *= us[2 * j];
                    u1 *= us[2 * j + 1];
                  }
                  packed[j] = pack2<TOUT>(silu_mul(g0, u0), silu_mul(g1, u1));
                }
                uint4* dst = reinterpret_cast<uint4*>(out_row + g * 16);
                dst[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
                dst[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
              }
            }
          }
        }
      } else {
        constexpr int C_HALF = BN / 32;              // 16-column chunks per half
        constexpr int CPI = C_HALF >= 4 ? 4 : C_HALF;  // chunks per TMEM wait
        // a 128-column tail item: 4 chunks per column half
        const int c_half = c.half >= 0 ? 4 : C_HALF;
        const float w =
            valid ? load_weight(p.row_weights, p.row_weights_dtype, r) : 0.0f;
        // weighted rows in fp32 (K-split partial sums) or the activation dtype
        TOUT* out_row = static_cast<TOUT*>(p.out) +
                        (int64_t(c.ks) * p.numel + (valid ? r : 0)) * p.out_ld + col0;
#pragma unroll 1
        for (int cc = 0; cc < c_half; cc += CPI) {
          uint32_t v[CPI][16];
#pragma unroll
          for (int u = 0; u < CPI; ++u) tmem_ld16(tbase + (h * c_half + cc + u) * 16, v[u]);
          tmem_ld_wait();
          if (valid) {
#pragma unroll
            for (int u = 0; u < CPI; ++u) {
              const int g = h * c_half + cc + u;
              float x[16];
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                float s4[4] = {w, w, w, w};
                if constexpr (kScaled) {
                  const float s = a_s * w;
                  const float4 b4 = __ldg(reinterpret_cast<const float4*>(bsc + g * 16) + j);
                  s4[0] = s * b4.x;
                  s4[1] = s * b4.y;
                  s4[2] = s * b4.z;
                  s4[3] = s * b4.w;
                }
#pragma unroll
                for (int q2 = 0; q2 < 4; ++q2)
                  x[4 * j + q2] = acc_to_f32<KIND>(v[u][4 * j + q2]) * s4[q2];
              }
              if constexpr (std::is_same<TOUT, float>::value) {
                float4* dst = reinterpret_cast<float4*>(out_row + g * 16);
#pragma unroll
                for (int j = 0; j < 4; ++j)
                  dst[j] = make_float4(x[4 * j], x[4 * j + 1], x[4 * j + 2], x[4 * j + 3]);
              } else {
                uint4* dst = reinterpret_cast<uint4*>(out_row + g * 16);
#pragma unroll
                for (int j = 0; j < 2; ++j)
                  dst[j] = make_uint4(pack2<TOUT>(x[8 * j], x[8 * j + 1]),
                                      pack2<TOUT>(x[8 * j + 2], x[8 * j + 3]),
                                      pack2<TOUT>(x[8 * j + 4], x[8 * j + 5]),
                                      pack2<TOUT>(x[8 * j + 6], x[8 * j + 7]));
              }
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
  }

  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
  if (threadIdx.x == 0 && *abort_flag) report_status(p.status, MOE_ERR_TIMEOUT);
}


// ---------------------------------------------------------------------------
// FP8 (e4m3) block-scaled variant.
//
// The scales change every 128 elements of K (per token for A, per 128x128
// block for B), so the products of one k-block cannot be summed in TMEM
// across k-blocks. Each k-block is accumulated into a fresh TMEM buffer and
// sixteen epilogue warps promote it into fp32 registers:
//   acc[m, n] += a_scale[m, kb] * b_scale[e, n / 128, kb] * P_kb[m, n]
// TMEM holds 512 / BN such buffers (4 at BN = 128), so the MMAs of the next
// k-blocks run while one is promoted; each epilogue warp copies its columns
// out in 16-column batches (one batch of 32 at BN = 128) and releases the
// buffer as soon as the last batch is in registers, before its arithmetic.
// Warp w (4..19) owns TMEM lane quarter w % 4 and column quarter (w - 4) / 4
// (four warps per SM sub-partition hide the TMEM load latency);
// warps whose 32 rows are all padding skip the arithmetic.
// After the last k-block the gate-up epilogue applies SiLU(gate)*up and
// writes bf16 activations; the down epilogue scales by the top-k weight and
// writes fp32 rows.
// ---------------------------------------------------------------------------
// Warps 0-3 form the control warpgroup (TMA producer, MMA issuer, two idle
// warps); warps 4-19 are the epilogue. The block launches at kLaunchRegsF8
// registers per thread; the control warpgroup then gives registers back and
// the epilogue warpgroups take them (setmaxnreg), so the split must add up to
// the launch total exactly, which the host checks before the first launch.
constexpr int kEpiWarpsF8 = 16;
constexpr int kThreadsF8 = 128 + 32 * kEpiWarpsF8;
constexpr int kLaunchRegsF8 = 96;
constexpr int kCtrlRegsF8 = 32;
constexpr int kEpiRegsF8 = 112;
static_assert(128 * kCtrlRegsF8 + 32 * kEpiWarpsF8 * kEpiRegsF8 == kThreadsF8 * kLaunchRegsF8,
              "setmaxnreg split must equal the launch allocation");

template <int BN>
struct Fp8Cfg {
  static constexpr int kBufs = 512 / BN;  // TMEM partial buffers
  static constexpr int kHalf = BN / 4;    // columns per epilogue warp
  // columns per TMEM wait
  static constexpr int kBatch = kHalf > 32 ? 16 : kHalf;
};

// Each epilogue warp holds BN / 4 fp32 accumulators per thread (64 at
// BN = 256) plus one 16-column TMEM batch, within its 112 registers.
template <int BN, int EPI>
__global__ void __launch_bounds__(kThreadsF8, 1)
    moe_grouped_gemm_fp8_kernel(const __grid_constant__ CUtensorMap tmA,
                                const __grid_constant__ CUtensorMap tmB,
                                const KParams p) {
  using Cfg = GemmCfg<BN>;
  using F = Fp8Cfg<BN>;
  constexpr int STAGES = Cfg::kStages;
  constexpr int NBUF = F::kBufs;
  constexpr int HALF = F::kHalf;
  constexpr int BATCH = F::kBatch;
  constexpr uint32_t IDESC = make_idesc(1u, 0u, BM, BN);  // f32 <- e4m3 x e4m3
  static_assert(NBUF * BN == 512 && HALF % BATCH == 0 && BATCH % 16 == 0, "fp8 tiling");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + STAGES * kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * Cfg::kBBytes);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + NBUF;
  uint64_t* final_bar = tempty + NBUF;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(final_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < NBUF; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 32 * kEpiWarpsF8);
    }
    mbar_init(final_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // Programmatic dependent launch: without early metadata every thread
  // waits for the previous kernel here; with it, the align outputs are read
  // first (they were written two launches earlier), and only the A loads
  // (and so everything downstream of them) wait, after the first weight
  // tiles have been requested.
  const bool producer = warp == 0 && lane == 0;
  if (!p.early_meta) {
    pdl_wait();
    pdl_trigger();
  }
  const int num_mb = min(__ldg(p.num_post_pad) / BM, p.max_m_blocks);
  const int n_tiles = p.n_total / BN;
  const int total_tiles = num_mb * n_tiles * p.splits;
  const uint64_t limit = p.wait_limit_ns;
  uint32_t* gtab = reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(full) + 256);
  const bool use_tab = num_mb <= kMaxTableMb;
  if (use_tab)
    build_group_table(p.expert_ids, num_mb, gtab, reinterpret_cast<int*>(gtab + kMaxTableMb));
  auto coord = [&](int t) {
    return use_tab ? tile_coord_tab(t, n_tiles, p.splits, gtab)
                   : tile_coord(t, num_mb, n_tiles, p.splits);
  };
  if (p.early_meta && !producer) {
    pdl_wait();
    pdl_trigger();
  }

  if (warp < 4) setmaxnreg_dec<kCtrlRegsF8>();
  if (producer) {
    // ---------------- TMA producer ----------------
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    // early weight tiles, as in the bf16/int8 kernel
    uint32_t pre = 0;
    if (p.early_meta) {
      for (int t = blockIdx.x; pre < uint32_t(STAGES) && t < total_tiles; t += gridDim.x) {
        const TileCoord c = coord(t);
        const int e = __ldg(p.expert_ids + c.mb);
        if (e < 0 || e >= p.num_experts) continue;
        const int kb0 = c.ks * p.kb_per_split;
        const int kb1 = min(kb0 + p.kb_per_split, p.k_blocks);
        const int b_row = e * p.n_total + c.nt * BN;
        for (int kb = kb0; kb < kb1 && pre < uint32_t(STAGES); ++kb, ++pre) {
          mbar_arrive_expect_tx(&full[pre], Cfg::kStageBytes);
          tma_load_2d(sB + pre * Cfg::kBBytes, &tmB, kb * kKBytes, b_row, &full[pre]);
        }
      }
      pdl_wait();
      pdl_trigger();
    }
    int stage = 0;
    uint32_t phase = 0;
    uint32_t issued = 0;
    bool ok = true;
    for (int t = blockIdx.x; ok && t < total_tiles; t += gridDim.x) {
      const TileCoord c = coord(t);
      const int e = __ldg(p.expert_ids + c.mb);
      if (e < 0 || e >= p.num_experts) continue;
      const int kb0 = c.ks * p.kb_per_split;
      const int kb1 = min(kb0 + p.kb_per_split, p.k_blocks);
      const int a_row = c.mb * BM;
      const int b_row = e * p.n_total + c.nt * BN;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (issued < pre) {
          tma_load_2d(sA + stage * kABytes, &tmA, kb * kKBytes, a_row, &full[stage]);
        } else {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1u, abort_flag, limit)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], Cfg::kStageBytes);
          tma_load_2d(sA + stage * kABytes, &tmA, kb * kKBytes, a_row, &full[stage]);
          tma_load_2d(sB + stage * Cfg::kBBytes, &tmB, kb * kKBytes, b_row, &full[stage]);
        }
        ++issued;
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    for (int s = 0; s < STAGES; ++s) {
      const uint32_t n_s = issued / STAGES + (uint32_t(s) < issued % STAGES ? 1u : 0u);
      if (n_s == 0) continue;
      volatile int no_abort = 0;
      mbar_wait_bounded(&full[s], (n_s - 1) & 1u, &no_abort, limit);
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer: one TMEM buffer per k-block ----------------
    int stage = 0;
    uint32_t phase = 0;
    int pb = 0;
    uint32_t pphase = 0;
    bool ok = true;
    for (int t = blockIdx.x; ok && t < total_tiles; t += gridDim.x) {
      const TileCoord c = coord(t);
      const int e = __ldg(p.expert_ids + c.mb);
      if (e < 0 || e >= p.num_experts) continue;
      const int kb0 = c.ks * p.kb_per_split;
      const int kb1 = min(kb0 + p.kb_per_split, p.k_blocks);
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait_bounded(&tempty[pb], pphase ^ 1u, abort_flag, limit) ||
            !mbar_wait_bounded(&full[stage], phase, abort_flag, limit)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + uint32_t(pb * BN);
        const uint32_t a0 = smem_u32(sA + stage * kABytes);
        const uint32_t b0 = smem_u32(sB + stage * Cfg::kBBytes);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          tc_mma<kKindF8>(d_tmem, make_sw128_desc(a0 + kk * 32), make_sw128_desc(b0 + kk * 32),
                          IDESC, kk > 0 ? 1u : 0u);
        tc_commit(&empty[stage]);
        tc_commit(&tfull[pb]);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
        if (++pb == NBUF) {
          pb = 0;
          pphase ^= 1u;
        }
      }
    }
    tc_commit(final_bar);
    volatile int no_abort = 0;
    mbar_wait_bounded(final_bar, 0, &no_abort, limit);
  } else if (warp >= 4) {
    // ---------------- promotion + epilogue (16 warps) ----------------
    setmaxnreg_inc<kEpiRegsF8>();
    const int q = warp & 3;
    const int h = (warp - 4) >> 2;
    const int row = q * 32 + lane;
    const int col0 = h * HALF;
    int pb = 0;
    uint32_t pphase = 0;
    bool aborted = false;
    for (int t = blockIdx.x; !aborted && t < total_tiles; t += gridDim.x) {
      const TileCoord c = coord(t);
      const int e = __ldg(p.expert_ids + c.mb);
      if (e < 0 || e >= p.num_experts) continue;
      const int kb0 = c.ks * p.kb_per_split;
      const int kb1 = min(kb0 + p.kb_per_split, p.k_blocks);
      const int m = c.mb * BM + row;
      const int r = __ldg(p.sorted_ids + m);
      const bool valid = r < p.numel;
      const bool warp_live = __any_sync(0xffffffffu, valid);
      const int n0 = c.nt * BN + col0;  // first output column of this half
      int rb0, rb1;
      if constexpr (EPI == kEpiSwiGLU) {
        rb0 = (16 * (n0 / 32)) / 128;                 // gate rows' block
        rb1 = (p.up_offset + 16 * (n0 / 32)) / 128;   // up rows' block
      } else {
        rb0 = n0 / 128;
        rb1 = rb0;
      }
      const float* sb0 = p.b_scale + (int64_t(e) * p.sb_rb + rb0) * p.sb_kb;
      const float* sb1 = p.b_scale + (int64_t(e) * p.sb_rb + rb1) * p.sb_kb;
      const float* sap = p.a_scale + int64_t(m) * p.sa_ld;
      float acc[HALF];
#pragma unroll
      for (int j = 0; j < HALF; ++j) acc[j] = 0.0f;
      // scales of the next k-block are loaded one step ahead, so their
      // latency hides behind the barrier wait and the TMEM copy
      float sa_n = valid ? __ldg(sap + kb0) : 0.0f;
      float sb0_n = __ldg(sb0 + kb0);
      float sb1_n = __ldg(sb1 + kb0);
      for (int kb = kb0; kb < kb1; ++kb) {
        const float s0 = sa_n * sb0_n;
        const float s1 = sa_n * sb1_n;
        if (kb + 1 < kb1) {
          sa_n = valid ? __ldg(sap + kb + 1) : 0.0f;
          sb0_n = __ldg(sb0 + kb + 1);
          sb1_n = __ldg(sb1 + kb + 1);
        }
        const bool ok = mbar_wait_bounded(&tfull[pb], pphase, abort_flag, limit);
        if (!__all_sync(0xffffffffu, ok)) {
          aborted = true;
          break;
        }
        tc_fence_after();
        const uint32_t tbase =
            tmem_base + (uint32_t(q * 32) << 16) + uint32_t(pb * BN + col0);
#pragma unroll
        for (int b0 = 0; b0 < HALF; b0 += BATCH) {
          uint32_t v[BATCH];
#pragma unroll
          for (int u = 0; u < BATCH / 16; ++u)
            tmem_ld16(tbase + b0 + 16 * u, *reinterpret_cast<uint32_t(*)[16]>(&v[16 * u]));
          tmem_ld_wait();
          if (b0 + BATCH >= HALF) {
            // every column of this buffer is in registers: hand it back
            tc_fence_before();
            mbar_arrive(&tempty[pb]);
          }
          if (warp_live) {
#pragma unroll
            for (int j = 0; j < BATCH; ++j) {
              // a 32-column group holds 16 gate columns then 16 up columns
              const float sc = (EPI == kEpiSwiGLU && ((b0 + j) & 31) >= 16) ? s1 : s0;
              acc[b0 + j] = fmaf(sc, __uint_as_float(v[j]), acc[b0 + j]);
            }
          }
        }
        if (++pb == NBUF) {
          pb = 0;
          pphase ^= 1u;
        }
      }
      if (aborted || !valid) continue;
      if constexpr (EPI == kEpiSwiGLU) {
        __nv_bfloat16* out_row =
            static_cast<__nv_bfloat16*>(p.out) + int64_t(m) * p.out_ld + n0 / 2;
#pragma unroll
        for (int gi = 0; gi < HALF / 32; ++gi) {
          uint32_t packed[8];
#pragma unroll
          for (int j = 0; j < 8; ++j)
            packed[j] = pack2<__nv_bfloat16>(
                silu_mul(acc[gi * 32 + 2 * j], acc[gi * 32 + 16 + 2 * j]),
                silu_mul(acc[gi * 32 + 2 * j + 1], acc[gi * 32 + 16 + 2 * j + 1]));
          uint4* dst = reinterpret_cast<uint4*>(out_row + gi * 16);
          dst[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
          dst[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
        }
      } else {
        const float w = load_weight(p.row_weights, p.row_weights_dtype, r);
        float* out_row =
            static_cast<float*>(p.out) + (int64_t(c.ks) * p.numel + r) * p.out_ld + n0;
#pragma unroll
        for (int j = 0; j < HALF; j += 4)
          *reinterpret_cast<float4*>(out_row + j) =
              make_float4(w * acc[j], w * acc[j + 1], w * acc[j + 2], w * acc[j + 3]);
      }
    }
  }

  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
  if (threadIdx.x == 0 && *abort_flag) report_status(p.status, MOE_ERR_TIMEOUT);
}

// ---------------------------------------------------------------------------
// FP8 (e4m3) with power-of-two (UE8M0) block scales applied by the tensor
// core: tcgen05.mma kind::mxf8f6f4.block_scale takes, for every K = 32 step,
// one scale byte per A row and per B row from tensor memory, so all k-blocks
// of a tile accumulate in one TMEM buffer as in the bf16 kernel, and the
// epilogue is the bf16 kernel's (no per-k-block promotion).
//
// Per k-block the producer also brings the 512-byte scale-factor chunk of
// the A tile's 128 rows and the BN / 128 chunks of the B tile (bulk copies
// from the scale-factor images into the stage). The MMA thread copies them
// into the stage's TMEM slot (tcgen05.cp; copies and MMAs issued by one
// thread execute in order) and selects byte kb % 4 of each 32-bit cell
// through the instruction descriptor. A slot is rewritten only after the
// MMAs that read it have completed (the stage went through its empty
// barrier first). A BN = 256 tile keeps one accumulator (its 256 columns and
// the scale slots share the 512 TMEM columns), BN = 128 two.
//
// Image geometry (the moe_ue8m0_scale_bytes layout): A has rows / 128 row
// slices and ceil(k_blocks / 4) chunk columns; B has n_total / 128 row
// slices per expert.
// ---------------------------------------------------------------------------
template <int BN>
struct MxCfg {
  static constexpr int kNAcc = BN == 256 ? 1 : 2;
  static constexpr int kBBytes = BN * kKBytes;
  static constexpr int kSfaBytes = 512;
  static constexpr int kSfbBytes = (BN / 128) * 512;
  static constexpr int kStageBytes = kABytes + kBBytes + kSfaBytes + kSfbBytes;
  static constexpr size_t kFixedBytes = 1024 + 256 + kGroupTableBytes;
  static constexpr int kStages = int((224 * 1024 - kFixedBytes) / kStageBytes);
  static constexpr size_t kSmemBytes = kFixedBytes + size_t(kStages) * kStageBytes;
  static constexpr int kSfCol0 = kNAcc * BN;          // first scale-slot column
  static constexpr int kSfCols = 4 + 4 * (BN / 128);  // A chunk + B chunks per stage
  static_assert(BN == 128 || BN == 256, "block-scaled tile width");
  static_assert(kStages >= 2 && 8 * (2 * kStages + 5) + 8 <= 256, "pipeline depth");
  static_assert(kSfCol0 + kStages * kSfCols <= 512, "TMEM columns");
};

// Block-scaled MMAs exist with M = 128 only (one CTA), so every m-block runs
// full-height tiles here, padding rows included.
template <int BN, int EPI, typename TOUT>
__global__ void __launch_bounds__(kThreads, 1)
    moe_grouped_gemm_mx_kernel(const __grid_constant__ CUtensorMap tmA,
                               const __grid_constant__ CUtensorMap tmB, const KParams p) {
  using Cfg = MxCfg<BN>;
  constexpr int STAGES = Cfg::kStages;
  constexpr int NACC = Cfg::kNAcc;
  constexpr uint32_t IDESC = make_idesc_mx(BM, BN);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + STAGES * kABytes;
  uint8_t* sSfa = sB + STAGES * Cfg::kBBytes;
  uint8_t* sSfb = sSfa + STAGES * Cfg::kSfaBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sSfb + STAGES * Cfg::kSfbBytes);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* final_bar = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(final_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < NACC; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 256);
    }
    mbar_init(final_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // programmatic dependent launch, as in moe_grouped_gemm_kernel
  const bool producer = warp == 0 && lane == 0;
  if (!p.early_meta) {
    pdl_wait();
    pdl_trigger();
  }
  const int num_mb = min(__ldg(p.num_post_pad) / BM, p.max_m_blocks);
  const int n_tiles = p.n_total / BN;
  const int total_tiles = num_mb * n_tiles * p.splits;
  const uint64_t limit = p.wait_limit_ns;
  uint32_t* gtab = reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(full) + 256);
  const bool use_tab = num_mb <= kMaxTableMb;
  if (use_tab)
    build_group_table(p.expert_ids, num_mb, gtab, reinterpret_cast<int*>(gtab + kMaxTableMb));
  auto coord = [&](int t) {
    return use_tab ? tile_coord_tab(t, n_tiles, p.splits, gtab)
                   : tile_coord(t, num_mb, n_tiles, p.splits);
  };
  if (p.early_meta && !producer) {
    pdl_wait();
    pdl_trigger();
  }

  if (producer) {
    // ---------------- TMA + scale-factor producer ----------------
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    const uint8_t* sfa_img = reinterpret_cast<const uint8_t*>(p.a_scale);
    const uint8_t* sfb_img = reinterpret_cast<const uint8_t*>(p.b_scale);
    const int64_t q_blocks = (p.k_blocks + 3) / 4;
    const int64_t b_slices = p.n_total / 128;
    auto sfa_src = [&](int mb, int kb) {
      return sfa_img + (int64_t(kb >> 2) * p.max_m_blocks + mb) * 512;
    };
    auto sfb_src = [&](int e, int nt, int kb) {
      return sfb_img + ((int64_t(e) * q_blocks + (kb >> 2)) * b_slices + nt * (BN / 128)) * 512;
    };
    uint32_t pre = 0;
    if (p.early_meta) {
      for (int t = blockIdx.x; pre < uint32_t(STAGES) && t < total_tiles; t += gridDim.x) {
        const TileCoord c = coord(t);
        const int e = __ldg(p.expert_ids + c.mb);
        if (e < 0 || e >= p.num_experts) continue;
        const int kb0 = c.ks * p.kb_per_split;
        const int kb1 = min(kb0 + p.kb_per_split, p.k_blocks);
        const int b_row = e * p.n_total + c.nt * BN;
        for (int kb = kb0; kb < kb1 && pre < uint32_t(STAGES); ++kb, ++pre) {
          mbar_arrive_expect_tx(&full[pre], Cfg::kStageBytes);
          tma_load_2d(sB + pre * Cfg::kBBytes, &tmB, kb * kKBytes, b_row, &full[pre]);
          bulk_load(sSfb + pre * Cfg::kSfbBytes, sfb_src(e, c.nt, kb), Cfg::kSfbBytes,
                    &full[pre]);
        }
      }
      pdl_wait();
      pdl_trigger();
    }
    int stage = 0;
    uint32_t phase = 0;
    uint32_t issued = 0;
    bool ok = true;
    for (int t = blockIdx.x; ok && t < total_tiles; t += gridDim.x) {
      const TileCoord c = coord(t);
      const int e = __ldg(p.expert_ids + c.mb);
      if (e < 0 || e >= p.num_experts) continue;
      const int kb0 = c.ks * p.kb_per_split;
      const int kb1 = min(kb0 + p.kb_per_split, p.k_blocks);
      const int a_row = c.mb * BM;
      const int b_row = e * p.n_total + c.nt * BN;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (issued >= pre) {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1u, abort_flag, limit)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], Cfg::kStageBytes);
          tma_load_2d(sB + stage * Cfg::kBBytes, &tmB, kb * kKBytes, b_row, &full[stage]);
          bulk_load(sSfb + stage * Cfg::kSfbBytes, sfb_src(e, c.nt, kb), Cfg::kSfbBytes,
                    &full[stage]);
        }
        tma_load_2d(sA + stage * kABytes, &tmA, kb * kKBytes, a_row, &full[stage]);
        bulk_load(sSfa + stage * Cfg::kSfaBytes, sfa_src(c.mb, kb), Cfg::kSfaBytes,
                  &full[stage]);
        ++issued;
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    for (int s = 0; s < STAGES; ++s) {
      const uint32_t n_s = issued / STAGES + (uint32_t(s) < issued % STAGES ? 1u : 0u);
      if (n_s == 0) continue;
      volatile int no_abort = 0;
      mbar_wait_bounded(&full[s], (n_s - 1) & 1u, &no_abort, limit);
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------- scale-factor copies + MMA issuer ----------------
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    for (int t = blockIdx.x; ok && t < total_tiles; t += gridDim.x) {
      const TileCoord c = coord(t);
      const int e = __ldg(p.expert_ids + c.mb);
      if (e < 0 || e >= p.num_experts) continue;
      const int kb0 = c.ks * p.kb_per_split;
      const int kb1 = min(kb0 + p.kb_per_split, p.k_blocks);
      if (!mbar_wait_bounded(&tempty[acc], acc_phase ^ 1u, abort_flag, limit)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + uint32_t(acc * BN);
      const uint32_t idesc_tile = IDESC;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait_bounded(&full[stage], phase, abort_flag, limit)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sf_t = tmem_base + uint32_t(Cfg::kSfCol0 + stage * Cfg::kSfCols);
        tc_cp_sf(sf_t, make_sf_desc(smem_u32(sSfa + stage * Cfg::kSfaBytes)));
#pragma unroll
        for (int j = 0; j < BN / 128; ++j)
          tc_cp_sf(sf_t + 4 + 4 * j,
                   make_sf_desc(smem_u32(sSfb + stage * Cfg::kSfbBytes + 512 * j)));
        const uint32_t idesc = idesc_sf_ids(idesc_tile, uint32_t(kb & 3));
        const uint32_t a0 = smem_u32(sA + stage * kABytes);
        const uint32_t b0 = smem_u32(sB + stage * Cfg::kBBytes);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          tc_mma_mx(d_tmem, make_sw128_desc(a0 + kk * 32), make_sw128_desc(b0 + kk * 32),
                    idesc, sf_t, sf_t + 4, (kb > kb0 || kk > 0) ? 1u : 0u);
        tc_commit(&empty[stage]);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) break;
      tc_commit(&tfull[acc]);
      if (++acc == NACC) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    tc_commit(final_bar);
    volatile int no_abort = 0;
    mbar_wait_bounded(final_bar, 0, &no_abort, limit);
  } else if (warp >= 2) {
    // ---------------- epilogue (8 warps), as in moe_grouped_gemm_kernel ----------------
    const int q = warp & 3;
    const int h = (warp - 2) >> 2;
    const int row = q * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < total_tiles; t += gridDim.x) {
      const TileCoord c = coord(t);
      const int e = __ldg(p.expert_ids + c.mb);
      if (e < 0 || e >= p.num_experts) continue;
      bool ok = mbar_wait_bounded(&tfull[acc], acc_phase, abort_flag, limit);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      const int m = c.mb * BM + row;
      const int r = __ldg(p.sorted_ids + m);
      const bool valid = r < p.numel;
      const uint32_t tbase = tmem_base + (uint32_t(q * 32) << 16) + uint32_t(acc * BN);
      if constexpr (EPI == kEpiSwiGLU) {
        constexpr int G_HALF = BN / 64;
        constexpr int GPI = G_HALF >= 2 ? 2 : 1;
        TOUT* out_row = static_cast<TOUT*>(p.out) + int64_t(m) * p.out_ld + c.nt * (BN / 2);
#pragma unroll 1
        for (int gg = 0; gg < G_HALF; gg += GPI) {
          uint32_t gv[GPI][16], uv[GPI][16];
#pragma unroll
          for (int u = 0; u < GPI; ++u) {
            const int g = h * G_HALF + gg + u;
            tmem_ld16(tbase + g * 32, gv[u]);
            tmem_ld16(tbase + g * 32 + 16, uv[u]);
          }
          tmem_ld_wait();
          if (valid) {
#pragma unroll
            for (int u = 0; u < GPI; ++u) {
              const int g = h * G_HALF + gg + u;
              uint32_t packed[8];
#pragma unroll
              for (int j = 0; j < 8; ++j)
                packed[j] = pack2<TOUT>(
                    silu_mul(__uint_as_float(gv[u][2 * j]), __uint_as_float(uv[u][2 * j])),
                    silu_mul(__uint_as_float(gv[u][2 * j + 1]),
                             __uint_as_float(uv[u][2 * j + 1])));
              uint4* dst = reinterpret_cast<uint4*>(out_row + g * 16);
              dst[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
              dst[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
            }
          }
        }
      } else {
        constexpr int C_HALF = BN / 32;
        constexpr int CPI = C_HALF >= 4 ? 4 : C_HALF;
        const float w = valid ? load_weight(p.row_weights, p.row_weights_dtype, r) : 0.0f;
        TOUT* out_row = static_cast<TOUT*>(p.out) +
                        (int64_t(c.ks) * p.numel + (valid ? r : 0)) * p.out_ld + c.nt * BN;
#pragma unroll 1
        for (int cc = 0; cc < C_HALF; cc += CPI) {
          uint32_t v[CPI][16];
#pragma unroll
          for (int u = 0; u < CPI; ++u) tmem_ld16(tbase + (h * C_HALF + cc + u) * 16, v[u]);
          tmem_ld_wait();
          if (valid) {
#pragma unroll
            for (int u = 0; u < CPI; ++u) {
              const int g = h * C_HALF + cc + u;
              float x[16];
#pragma unroll
              for (int j = 0; j < 16; ++j) x[j] = __uint_as_float(v[u][j]) * w;
              if constexpr (std::is_same<TOUT, float>::value) {
                float4* dst = reinterpret_cast<float4*>(out_row + g * 16);
#pragma unroll
                for (int j = 0; j < 4; ++j)
                  dst[j] = make_float4(x[4 * j], x[4 * j + 1], x[4 * j + 2], x[4 * j + 3]);
              } else {
                uint4* dst = reinterpret_cast<uint4*>(out_row + g * 16);
#pragma unroll
                for (int j = 0; j < 2; ++j)
                  dst[j] = make_uint4(pack2<TOUT>(x[8 * j], x[8 * j + 1]),
                                      pack2<TOUT>(x[8 * j + 2], x[8 * j + 3]),
                                      pack2<TOUT>(x[8 * j + 4], x[8 * j + 5]),
                                      pack2<TOUT>(x[8 * j + 6], x[8 * j + 7]));
              }
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
      if (++acc == NACC) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  }

  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
  if (threadIdx.x == 0 && *abort_flag) report_status(p.status, MOE_ERR_TIMEOUT);
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

int num_sms_or_fail(int* sms) { return check_device(sms); }

// Raises a kernel's dynamic shared-memory limit once per device (the
// attribute is per function and device; setting it on every launch costs
// host time on the decode path).
template <typename Kern>
int set_smem_once(Kern kern, size_t bytes, std::atomic<uint64_t>& done) {
  int dev = 0;
  KSW_CUDA(cudaGetDevice(&dev));
  const uint64_t bit = dev < 64 ? (uint64_t(1) << dev) : 0;
  if (bit && (done.load(std::memory_order_acquire) & bit)) return MOE_OK;
  KSW_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(bytes)));
  done.fetch_or(bit, std::memory_order_acq_rel);
  return MOE_OK;
}

template <int KIND, int AB_FMT, int BN, int EPI, typename TOUT>
int launch_kernel(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tb128,
                  const KParams& kp, int grid, cudaStream_t s) {
  using Cfg = GemmCfg<BN>;
  auto kern = moe_grouped_gemm_kernel<KIND, AB_FMT, BN, EPI, TOUT>;
  static std::atomic<uint64_t> smem_set{0};
  int st = set_smem_once(kern, Cfg::kSmemBytes, smem_set);
  if (st != MOE_OK) return st;
  KSW_LAUNCH(kern, dim3(grid), dim3(kThreads), Cfg::kSmemBytes, s, ta, tb, tb128, kp);
  return MOE_OK;
}

template <int BN, int EPI>
int launch_fp8(const CUtensorMap& ta, const CUtensorMap& tb, const KParams& kp, int grid,
               cudaStream_t s) {
  using Cfg = GemmCfg<BN>;
  auto kern = moe_grouped_gemm_fp8_kernel<BN, EPI>;
  static std::atomic<uint64_t> smem_set{0};
  int st = set_smem_once(kern, Cfg::kSmemBytes, smem_set);
  if (st != MOE_OK) return st;
  // The setmaxnreg split inside the kernel assumes this launch allocation;
  // with any other, the epilogue's register request could never be met.
  static std::atomic<int> regs_ok{0};
  if (!regs_ok.load(std::memory_order_acquire)) {
    cudaFuncAttributes attr{};
    KSW_CUDA(cudaFuncGetAttributes(&attr, kern));
    KSW_REQUIRE(attr.numRegs == kLaunchRegsF8, MOE_ERR_DEVICE,
                "fp8 GEMM: kernel built with an unexpected register count");
    regs_ok.store(1, std::memory_order_release);
  }
  KSW_LAUNCH(kern, dim3(grid), dim3(kThreadsF8), Cfg::kSmemBytes, s, ta, tb, kp);
  return MOE_OK;
}

template <int EPI>
int dispatch_fp8(int bn, const CUtensorMap& ta, const CUtensorMap& tb, const KParams& kp,
                 int grid, cudaStream_t s) {
  switch (bn) {
    case 256: return launch_fp8<256, EPI>(ta, tb, kp, grid, s);
    case 128: return launch_fp8<128, EPI>(ta, tb, kp, grid, s);
    default: return fail(MOE_ERR_UNSUPPORTED, "fp8 GEMM: block_n must be 128 or 256");
  }
}

template <int BN, int EPI, typename TOUT>
int launch_mx(const CUtensorMap& ta, const CUtensorMap& tb, const KParams& kp, int grid,
              cudaStream_t s) {
  using Cfg = MxCfg<BN>;
  auto kern = moe_grouped_gemm_mx_kernel<BN, EPI, TOUT>;
  static std::atomic<uint64_t> smem_set{0};
  int st = set_smem_once(kern, Cfg::kSmemBytes, smem_set);
  if (st != MOE_OK) return st;
  KSW_LAUNCH(kern, dim3(grid), dim3(kThreads), Cfg::kSmemBytes, s, ta, tb, kp);
  return MOE_OK;
}

template <int EPI, typename TOUT>
int dispatch_mx(int bn, const CUtensorMap& ta, const CUtensorMap& tb, const KParams& kp,
                int grid, cudaStream_t s) {
  switch (bn) {
    case 256: return launch_mx<256, EPI, TOUT>(ta, tb, kp, grid, s);
    case 128: return launch_mx<128, EPI, TOUT>(ta, tb, kp, grid, s);
    default: return fail(MOE_ERR_UNSUPPORTED, "fp8 ue8m0 GEMM: block_n must be 128 or 256");
  }
}

template <int KIND, int AB_FMT, int EPI, typename TOUT>
int dispatch_bn(int bn, const CUtensorMap& ta, const CUtensorMap& tb,
                const KParams& kp, int grid, cudaStream_t s,
                const CUtensorMap* tb128 = nullptr) {
  // tb128: the weights with 128-row boxes, for tail halves (kp.tail_halves)
  const CUtensorMap& t128 = tb128 != nullptr ? *tb128 : tb;
  switch (bn) {
    case 256: return launch_kernel<KIND, AB_FMT, 256, EPI, TOUT>(ta, tb, t128, kp, grid, s);
    case 128: return launch_kernel<KIND, AB_FMT, 128, EPI, TOUT>(ta, tb, t128, kp, grid, s);
    case 64: return launch_kernel<KIND, AB_FMT, 64, EPI, TOUT>(ta, tb, t128, kp, grid, s);
    default: return fail(MOE_ERR_UNSUPPORTED, "unsupported block_n");
  }
}

// Picks the N tile: the largest of 256/128/64 dividing n that still gives
// every SM about two tiles, given an upper bound on the m-blocks.
int pick_block_n(int64_t n, int64_t est_m_blocks, int64_t splits, int sms,
                 bool allow64 = true) {
  const int cands[3] = {256, 128, 64};
  int best = 0;
  for (int bn : cands) {
    if (bn == 64 && !allow64) break;
    if (n % bn != 0) continue;
    if (best == 0) best = bn;
    if (est_m_blocks * (n / bn) * splits >= 2 * int64_t(sms)) return bn;
    best = bn;
  }
  return best;
}

int common_checks(const GroupedGemmArgs& a) {
  KSW_REQUIRE(a.a && a.b && a.sorted_ids && a.expert_ids && a.num_post_pad && a.out,
              MOE_ERR_INVALID_ARG, "grouped GEMM: null pointer");
  // TMA operands, 16-byte epilogue stores, float4 / bulk-copied scales
  KSW_REQUIRE(aligned16(a.a) && aligned16(a.b) && aligned16(a.out) &&
                  (a.quant == MOE_QUANT_FP8_BLOCK ||
                   (aligned16(a.a_scale) && aligned16(a.b_scale))),
              MOE_ERR_INVALID_ARG, "grouped GEMM: operands must be 16-byte aligned");
  KSW_REQUIRE(a.rows > 0 && a.rows % BM == 0, MOE_ERR_INVALID_ARG,
              "grouped GEMM: rows must be a positive multiple of 128");
  KSW_REQUIRE(a.num_experts >= 1 && a.n > 0 && a.k > 0, MOE_ERR_INVALID_ARG,
              "grouped GEMM: bad sizes");
  KSW_REQUIRE(int64_t(a.num_experts) * a.n < (int64_t(1) << 31),
              MOE_ERR_UNSUPPORTED, "grouped GEMM: E * N too large");
  KSW_REQUIRE(a.rows < (int64_t(1) << 31) && a.numel < (int64_t(1) << 31),
              MOE_ERR_UNSUPPORTED, "grouped GEMM: too many rows");
  return MOE_OK;
}

struct OperandTypes {
  CUtensorMapDataType tma_type;
  int elem_bytes;
};

int operand_types(const GroupedGemmArgs& a, OperandTypes* ot) {
  if (a.quant == MOE_QUANT_NONE && a.compute_dtype == MOE_DTYPE_F32) {
    // fp32 operands, multiplied as tf32 (kind::tf32)
    ot->tma_type = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    ot->elem_bytes = 4;
    return MOE_OK;
  }
  if (a.quant == MOE_QUANT_NONE) {
    KSW_REQUIRE(a.compute_dtype == MOE_DTYPE_BF16 || a.compute_dtype == MOE_DTYPE_F16,
                MOE_ERR_INVALID_ARG, "compute dtype must be bf16, f16 or f32");
    ot->tma_type = a.compute_dtype == MOE_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                     : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    ot->elem_bytes = 2;
    return MOE_OK;
  }
  if (a.quant == MOE_QUANT_INT8_CHANNEL || a.quant == MOE_QUANT_FP8_BLOCK ||
      a.quant == MOE_QUANT_FP8_UE8M0) {
    KSW_REQUIRE(a.a_scale && a.b_scale, MOE_ERR_INVALID_ARG,
                "W8A8 GEMM needs activation and weight scales");
    ot->tma_type = CU_TENSOR_MAP_DATA_TYPE_UINT8;
    ot->elem_bytes = 1;
    return MOE_OK;
  }
  return fail(MOE_ERR_UNSUPPORTED, "quant mode not handled by this GEMM");
}

int make_maps(const GroupedGemmArgs& a, const OperandTypes& ot, int bn,
              CUtensorMap* ta, CUtensorMap* tb) {
  const uint32_t box_k = uint32_t(kKBytes / ot.elem_bytes);
  int st = encode_tma_2d(ta, ot.tma_type, ot.elem_bytes, a.a, uint64_t(a.k), uint64_t(a.rows),
                         uint64_t(a.k), box_k, uint32_t(BM));
  if (st != MOE_OK) return st;
  return encode_tma_2d(tb, ot.tma_type, ot.elem_bytes, a.b, uint64_t(a.k),
                       uint64_t(a.num_experts) * uint64_t(a.n), uint64_t(a.k),
                       box_k, uint32_t(bn));
}

// MOE_NO_TAIL_HALVES=1 runs every tile of the rows GEMMs at full width (the
// tests compare both; read once).
bool tail_halves_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("MOE_NO_TAIL_HALVES");
    return !(v && v[0] && v[0] != '0');
  }();
  return on;
}

KParams base_params(const GroupedGemmArgs& a, int elem_bytes) {
  KParams kp{};
  kp.num_post_pad = a.num_post_pad;
  kp.expert_ids = a.expert_ids;
  kp.sorted_ids = a.sorted_ids;
  kp.a_scale = a.a_scale;
  kp.b_scale = a.b_scale;
  kp.row_weights = a.row_weights;
  kp.out = a.out;
  kp.status = a.status;
  kp.max_m_blocks = int32_t(a.rows / BM);
  kp.n_total = int32_t(a.n);
  kp.k_blocks = int32_t(ceil_div(a.k * elem_bytes, kKBytes));
  kp.splits = 1;
  kp.kb_per_split = kp.k_blocks;
  kp.numel = int32_t(a.numel);
  kp.num_experts = a.num_experts;
  kp.row_weights_dtype = a.row_weights_dtype;
  kp.sa_ld = int32_t(ceil_div(a.k, 128));
  kp.sb_rb = int32_t(ceil_div(a.n, 128));
  kp.sb_kb = int32_t(ceil_div(a.k, 128));
  kp.up_offset = int32_t(a.n / 2);
  kp.early_meta = a.early_meta;
  kp.wait_limit_ns = kWaitLimitNs;
  return kp;
}

// Upper bound on the m-blocks actually used: every expert with rows adds at
// most one partial block.
int64_t est_m_blocks(const GroupedGemmArgs& a) {
  return std::min<int64_t>(a.rows / BM,
                           ceil_div(a.numel, BM) + std::min<int64_t>(a.num_experts, a.numel));
}

}  // namespace

int gemm_gate_up_launch(const GroupedGemmArgs& a, cudaStream_t s) {
  int sms = 0;
  int st = num_sms_or_fail(&sms);
  if (st != MOE_OK) return st;
  st = common_checks(a);
  if (st != MOE_OK) return st;
  KSW_REQUIRE(a.n % 32 == 0, MOE_ERR_UNSUPPORTED,
              "gate-up GEMM: 2*I must be a multiple of 32");
  OperandTypes ot;
  st = operand_types(a, &ot);
  if (st != MOE_OK) return st;
  KSW_REQUIRE((a.k * ot.elem_bytes) % 16 == 0, MOE_ERR_UNSUPPORTED,
              "gate-up GEMM: hidden size * element size must be a multiple of 16 B");
  const bool mx = a.quant == MOE_QUANT_FP8_UE8M0;
  const bool fp8 = a.quant == MOE_QUANT_FP8_BLOCK || mx;
  if (fp8)
    KSW_REQUIRE(a.n % 256 == 0, MOE_ERR_UNSUPPORTED,
                "fp8 gate-up GEMM: I must be a multiple of 128");
  if (mx)
    KSW_REQUIRE(a.k % 128 == 0, MOE_ERR_UNSUPPORTED,
                "fp8 ue8m0 gate-up GEMM: the hidden size must be a multiple of 128");
  const int bn = a.block_n ? a.block_n : pick_block_n(a.n, est_m_blocks(a), 1, sms, !fp8);
  KSW_REQUIRE(bn > 0 && a.n % bn == 0, MOE_ERR_UNSUPPORTED,
              "gate-up GEMM: 2*I must be a multiple of 64");
  CUtensorMap ta, tb;
  st = make_maps(a, ot, bn, &ta, &tb);
  if (st != MOE_OK) return st;
  KParams kp = base_params(a, ot.elem_bytes);
  kp.out_ld = a.n / 2;
  const int grid = sms;
  if (mx) return dispatch_mx<kEpiSwiGLU, __nv_bfloat16>(bn, ta, tb, kp, grid, s);
  if (fp8) return dispatch_fp8<kEpiSwiGLU>(bn, ta, tb, kp, grid, s);
  if (a.quant == MOE_QUANT_INT8_CHANNEL) {
    // int8 products dequantise to bf16 activations
    return dispatch_bn<kKindI8, 1, kEpiSwiGLU, __nv_bfloat16>(bn, ta, tb, kp, grid, s);
  }
  if (a.compute_dtype == MOE_DTYPE_F32)
    return dispatch_bn<kKindTF32, 2, kEpiSwiGLU, float>(bn, ta, tb, kp, grid, s);
  if (a.compute_dtype == MOE_DTYPE_BF16)
    return dispatch_bn<kKindF16, 1, kEpiSwiGLU, __nv_bfloat16>(bn, ta, tb, kp, grid, s);
  return dispatch_bn<kKindF16, 0, kEpiSwiGLU, __half>(bn, ta, tb, kp, grid, s);
}

// Gate-up GEMM split along K: writes unweighted fp32 partial rows
// part[s, r, :] (2I columns, regrouped order) for the flat row r of every
// valid operand row; swiglu_reduce then sums the splits and applies SiLU*up.
// Used when there are too few output tiles to fill the GPU (decode).
int gemm_gate_up_split_launch(const GroupedGemmArgs& a, cudaStream_t s) {
  GroupedGemmArgs d = a;
  d.row_weights = nullptr;
  d.row_weights_dtype = MOE_DTYPE_F32;
  return gemm_down_launch(d, s);
}

int gemm_down_launch(const GroupedGemmArgs& a, cudaStream_t s) {
  int sms = 0;
  int st = num_sms_or_fail(&sms);
  if (st != MOE_OK) return st;
  st = common_checks(a);
  if (st != MOE_OK) return st;
  KSW_REQUIRE(a.row_weights_dtype == MOE_DTYPE_F32 || a.row_weights_dtype == MOE_DTYPE_F16 ||
                  a.row_weights_dtype == MOE_DTYPE_BF16,
              MOE_ERR_INVALID_ARG, "down GEMM: row weights must be f32/f16/bf16");
  KSW_REQUIRE(a.splits >= 1, MOE_ERR_INVALID_ARG, "down GEMM: splits must be >= 1");
  OperandTypes ot;
  st = operand_types(a, &ot);
  if (st != MOE_OK) return st;
  KSW_REQUIRE((a.k * ot.elem_bytes) % 16 == 0, MOE_ERR_UNSUPPORTED,
              "down GEMM: intermediate size * element size must be a multiple of 16 B");
  KSW_REQUIRE(a.n % 64 == 0, MOE_ERR_UNSUPPORTED,
              "down GEMM: hidden size must be a multiple of 64");
  KParams kp = base_params(a, ot.elem_bytes);
  // K splits: every split gets at least one k-block; the effective count is
  // recomputed so that no split is empty.
  const int kb_per = int(ceil_div(kp.k_blocks, a.splits));
  kp.kb_per_split = kb_per;
  kp.splits = int(ceil_div(kp.k_blocks, kb_per));
  KSW_REQUIRE(kp.splits == a.splits, MOE_ERR_INVALID_ARG,
              "down GEMM: splits leaves an empty K range; choose splits so that every split has k-blocks");
  const bool fp8 = a.quant == MOE_QUANT_FP8_BLOCK;
  const bool mx = a.quant == MOE_QUANT_FP8_UE8M0;
  if (fp8 || mx)
    KSW_REQUIRE(a.n % 128 == 0, MOE_ERR_UNSUPPORTED,
                "fp8 down GEMM: hidden size must be a multiple of 128");
  if (mx)
    KSW_REQUIRE(a.k % 128 == 0, MOE_ERR_UNSUPPORTED,
                "fp8 ue8m0 down GEMM: the intermediate size must be a multiple of 128");
  const int bn = a.block_n ? a.block_n
                           : pick_block_n(a.n, est_m_blocks(a), kp.splits, sms, !(fp8 || mx));
  KSW_REQUIRE(bn > 0 && a.n % bn == 0, MOE_ERR_UNSUPPORTED, "down GEMM: bad block_n");
  CUtensorMap ta, tb;
  st = make_maps(a, ot, bn, &ta, &tb);
  if (st != MOE_OK) return st;
  kp.out_ld = a.n;
  const int grid = sms;
  // 256-wide unsplit tiles of the bf16/f16/tf32/int8 kernel may run the last
  // partial wave as 128-column halves (moe_grouped_gemm_kernel)
  CUtensorMap tb128 = tb;
  if (bn == 256 && kp.splits == 1 && !fp8 && !mx && tail_halves_enabled()) {
    st = encode_tma_2d(&tb128, ot.tma_type, ot.elem_bytes, a.b, uint64_t(a.k),
                       uint64_t(a.num_experts) * uint64_t(a.n), uint64_t(a.k),
                       uint32_t(kKBytes / ot.elem_bytes), 128);
    if (st != MOE_OK) return st;
    kp.tail_halves = 1;
  }
  KSW_REQUIRE(a.out_dtype == MOE_DTYPE_F32 || ((a.out_dtype == MOE_DTYPE_BF16 ||
                                                  a.out_dtype == MOE_DTYPE_F16) &&
                                                 kp.splits == 1 && !fp8),
              MOE_ERR_UNSUPPORTED,
              "down GEMM: 16-bit rows only without K split and without fp8");
  if (fp8) return dispatch_fp8<kEpiRows>(bn, ta, tb, kp, grid, s);
  if (mx) {
    if (a.out_dtype == MOE_DTYPE_BF16)
      return dispatch_mx<kEpiRows, __nv_bfloat16>(bn, ta, tb, kp, grid, s);
    if (a.out_dtype == MOE_DTYPE_F32) return dispatch_mx<kEpiRows, float>(bn, ta, tb, kp, grid, s);
    return fail(MOE_ERR_UNSUPPORTED, "down GEMM: fp8 ue8m0 rows are f32 or bf16");
  }
  if (a.out_dtype == MOE_DTYPE_BF16) {
    if (a.quant == MOE_QUANT_INT8_CHANNEL)
      return dispatch_bn<kKindI8, 1, kEpiRows, __nv_bfloat16>(bn, ta, tb, kp, grid, s, &tb128);
    if (a.compute_dtype == MOE_DTYPE_BF16)
      return dispatch_bn<kKindF16, 1, kEpiRows, __nv_bfloat16>(bn, ta, tb, kp, grid, s, &tb128);
    return fail(MOE_ERR_UNSUPPORTED, "down GEMM: bf16 rows need bf16 operands");
  }
  if (a.out_dtype == MOE_DTYPE_F16) {
    if (a.quant == MOE_QUANT_NONE && a.compute_dtype == MOE_DTYPE_F16)
      return dispatch_bn<kKindF16, 0, kEpiRows, __half>(bn, ta, tb, kp, grid, s, &tb128);
    return fail(MOE_ERR_UNSUPPORTED, "down GEMM: f16 rows need f16 operands");
  }
  if (a.quant == MOE_QUANT_INT8_CHANNEL)
    return dispatch_bn<kKindI8, 1, kEpiRows, float>(bn, ta, tb, kp, grid, s, &tb128);
  if (a.compute_dtype == MOE_DTYPE_F32)
    return dispatch_bn<kKindTF32, 2, kEpiRows, float>(bn, ta, tb, kp, grid, s, &tb128);
  if (a.compute_dtype == MOE_DTYPE_BF16)
    return dispatch_bn<kKindF16, 1, kEpiRows, float>(bn, ta, tb, kp, grid, s, &tb128);
  return dispatch_bn<kKindF16, 0, kEpiRows, float>(bn, ta, tb, kp, grid, s, &tb128);
}

}  // namespace ksw
