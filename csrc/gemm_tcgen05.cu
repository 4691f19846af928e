// Grouped "swap-AB" GEMM on the 5th-generation tensor cores (tcgen05 + TMEM),
// operands staged by TMA. One kernel serves every projection of the model:
//
//   out[row, f] = epilogue( sum_k X[row, k] * W[group, f, k] )
//
// The weight matrix is the MMA's A operand (M = 128 output features per
// tile) and the token rows are the B operand (N = 32..256 rows per tile), so
// the accumulator D^T[f, row] lives in TMEM with one feature per lane. A
// decode step with a handful of tokens per expert therefore pays for N = 32
// token columns, not for a 128-row M tile, and the kernel streams each
// expert's weight tile from HBM exactly once.
//
// Work units are (row block, feature tile). Row blocks come from a device
// list written by the MoE routing kernel (grouped mode: one or more blocks
// per expert, <= BN rows each) or are derived from a host row count (dense
// mode: a single group). Units are dealt round-robin to a persistent grid,
// or, in stream-K mode (opt-in, grouped GEMMs), each CTA takes an equal
// contiguous range of the units' k-iterations (see SegIter).
//
// Warp roles (192 threads): warp 0 = TMA producer, warp 1 = TMEM allocator
// + MMA issuer, warps 2..5 = epilogue (TMEM -> registers -> global). Smem
// stages are guarded by full/empty mbarriers; the TMEM accumulator by
// tmem_full (tcgen05.commit) / tmem_empty (epilogue arrivals).
//
// Epilogues: plain store (+ residual), SwiGLU over a gate/up accumulator
// pair (two A tiles per stage: gate rows and up rows of the same expert),
// per-row scale (routing weight), and optional peer stores: the same bf16
// tile is written to up to 8 peer-GPU buffers (NVLink P2P stores), after
// which the last CTA to finish raises a release flag on every peer. That is
// the fused attention->FFN hand-off of the o_proj GEMM.
//
// No cluster launch: every TMA load is issued per CTA and reads this GPU's memory.

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "gemm_tcgen05.h"

namespace afd {

constexpr int kBM = 128;        // output features per tile (MMA M)
constexpr int kBK = 64;         // K per pipeline stage (one 128-byte swizzle atom)
constexpr int kBoxRows = 32;    // token rows per TMA box
constexpr int kThreads = 192;
constexpr int kEpiWarps = 4;

// Two TMEM accumulator slots let the MMA warp start tile i+1 while the
// epilogue drains tile i; SwiGLU tiles hold a gate and an up accumulator, so
// BN = 256 SwiGLU keeps a single slot (512 columns).
template <bool SWIGLU, int BN, int STAGES>
struct GemmSmem {
  static constexpr int kABytes = kBM * kBK * 2;              // 16 KB
  static constexpr int kBBytes = BN * kBK * 2;               // BN x 128 B
  static constexpr int kStageBytes = kABytes * (SWIGLU ? 2 : 1) + kBBytes;
  static constexpr int kDataBytes = kStageBytes * STAGES;
  static constexpr int kSlots = (SWIGLU && BN > 128) ? 1 : 2;
  static constexpr int kAccCols = BN;                        // fp32 columns per accumulator
  static constexpr int kSlotCols = kAccCols * (SWIGLU ? 2 : 1);
  static constexpr int kUsedCols = kSlotCols * kSlots;
  static constexpr int kTmemCols = kUsedCols <= 32 ? 32 : kUsedCols <= 64 ? 64
                                   : kUsedCols <= 128 ? 128 : kUsedCols <= 256 ? 256 : 512;
  // epilogue staging: per warp 16 rows x 32 features bf16
  static constexpr int kStageOutBytes = kEpiWarps * 16 * 32 * 2;
  static constexpr int kRowIdBytes = BN * 4;                 // gathered rows of one block
  static constexpr int kScaleBytes = kEpiWarps * BN * 4;     // warp-private row scales
  static constexpr int kTotal = kDataBytes + kStageOutBytes + kRowIdBytes + kScaleBytes +
                                1024 /*align*/ + 256 /*barriers*/;
};

__device__ __forceinline__ int4 unit_block(const GemmArgs& a, int b) {
  if (a.blocks != nullptr) return a.blocks[b];
  int rs = b * a.block_n;
  int n = min(a.block_n, a.dense_rows - rs);
  return make_int4(rs, n, 0, 0);
}

__device__ __forceinline__ int total_tiles(const GemmArgs& a) {
  int nb = a.blocks != nullptr ? *a.num_blocks : (a.dense_rows + a.block_n - 1) / a.block_n;
  return nb * a.f_tiles;
}

// Unit u -> (tile, k split). Splits of one tile are tiles-apart so that they
// run on different CTAs at the same time.
struct Unit {
  int tile, split;
};
__device__ __forceinline__ Unit unit_of(int u, int tiles) { return {u % tiles, u / tiles}; }

// The k-ranges this CTA works on, in order: (tile, k0, k1) plus the tile's
// piece index and piece count. Round-robin mode: units (tile, split) dealt
// round-robin, `splits` equal K ranges per tile. Stream-K mode: the
// tiles x total_k k-iterations are cut into gridDim.x contiguous ranges of
// equal length (each at least one tile long), so every CTA streams the same
// number of weight tiles; a tile cut by a range boundary has two pieces,
// whose partial sums the later-finishing CTA adds in piece order.
struct SegIter {
  bool sk;
  long long u, hi;      // stream-K: next k-iteration, end of this CTA's range
  int units, tiles, total_k, k_iters, splits;
  __device__ SegIter(bool stream_k, int tiles_, int total_k_, int splits_)
      : sk(stream_k), tiles(tiles_), total_k(total_k_), splits(splits_) {
    k_iters = total_k / splits;
    units = tiles * splits;
    if (sk) {
      const long long U = (long long)tiles * total_k;
      u = U * blockIdx.x / gridDim.x;
      hi = U * (blockIdx.x + 1) / gridDim.x;
    } else {
      u = blockIdx.x;
      hi = units;
    }
  }
  __device__ bool next(int& tile, int& k0, int& k1, int& piece, int& pieces) {
    if (u >= hi) return false;
    if (sk) {
      tile = (int)(u / total_k);
      k0 = (int)(u % total_k);
      k1 = (int)min((long long)total_k, k0 + (hi - u));
      piece = k0 == 0 ? 0 : 1;
      pieces = (k0 == 0 && k1 == total_k) ? 1 : 2;
      u += k1 - k0;
    } else {
      const Unit un = unit_of((int)u, tiles);
      tile = un.tile;
      k0 = un.split * k_iters;
      k1 = k0 + k_iters;
      piece = un.split;
      pieces = splits;
      u += gridDim.x;
    }
    return true;
  }
};

__device__ __forceinline__ void epi_bar() {  // the 4 epilogue warps only
  asm volatile("bar.sync 1, 128;" ::: "memory");
}

// Fused MoE combine of output-feature tile ft (see GemmArgs::cmb_*), run by
// the 128 epilogue threads: 16 threads x 8 features cover the tile's 128
// features of one token; 8 tokens at a time. Same summation order and
// roundings as moe_combine_kernel.
__device__ void combine_feature_tile(const GemmArgs& a, int ft) {
  const int et = threadIdx.x - 64;
  const int col = ft * 128 + (et & 15) * 8;
  const int Hf = a.f_tiles * 128;
  for (int t = et >> 4; t < a.cmb_T; t += 8) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    // all row indices, then all rows, then the sums in j order (loads in flight)
    int r[16];
    uint4 v[16];
#pragma unroll
    for (int j = 0; j < 16; ++j)
      r[j] = j < a.cmb_topk ? a.cmb_inv[(size_t)t * a.cmb_topk + j] : -1;
#pragma unroll
    for (int j = 0; j < 16; ++j)
      v[j] = r[j] >= 0 ? __ldcg(reinterpret_cast<const uint4*>(a.out + (size_t)r[j] * a.ld_out + col))
                       : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      if (r[j] < 0) continue;
      const uint32_t* pv = &v[j].x;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float x0, x1;
        unpack_bf16x2(pv[e], x0, x1);
        acc[2 * e] += x0;
        acc[2 * e + 1] += x1;
      }
    }
    if (a.cmb_residual != nullptr) {
      const uint4 rv =
          *reinterpret_cast<const uint4*>(a.cmb_residual + (size_t)t * a.cmb_ld_res + col);
      const uint32_t* pr = &rv.x;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float r0, r1;
        unpack_bf16x2(pr[e], r0, r1);
        acc[2 * e] = round_bf16(acc[2 * e]) + r0;
        acc[2 * e + 1] = round_bf16(acc[2 * e + 1]) + r1;
      }
    }
    uint4 u;
    u.x = pack_bf16x2(acc[0], acc[1]);
    u.y = pack_bf16x2(acc[2], acc[3]);
    u.z = pack_bf16x2(acc[4], acc[5]);
    u.w = pack_bf16x2(acc[6], acc[7]);
    if (a.cmb_out != nullptr)
      *reinterpret_cast<uint4*>(a.cmb_out + (size_t)t * a.cmb_ld_out + col) = u;
    for (int sg = 0; sg < a.n_peers; ++sg)
      if (t >= a.cmb_seg_offsets[sg] && t < a.cmb_seg_offsets[sg + 1])
        *reinterpret_cast<uint4*>(
            a.peer_out[sg] + (size_t)(t - a.cmb_seg_offsets[sg] + a.peer_row_offset) * Hf + col) =
            u;
  }
}

template <bool SWIGLU, int BN, int STAGES>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_swapab_kernel(const __grid_constant__ CUtensorMap tmap_w,
                       const __grid_constant__ CUtensorMap tmap_x, const GemmArgs args) {
  using L = GemmSmem<SWIGLU, BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __nv_bfloat16* stage_out = reinterpret_cast<__nv_bfloat16*>(smem + L::kDataBytes);
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + L::kDataBytes + L::kStageOutBytes);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;      // [kSlots]
  uint64_t* tempty_bar = tfull_bar + 2;          // [kSlots]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty_bar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* rows_s = reinterpret_cast<int*>(smem + L::kDataBytes + L::kStageOutBytes + 256);
  float* scale_s = reinterpret_cast<float*>(smem + L::kDataBytes + L::kStageOutBytes + 256 +
                                            L::kRowIdBytes);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int s = 0; s < L::kSlots; ++s) {
      mbar_init(&tfull_bar[s], 1);
      mbar_init(&tempty_bar[s], kEpiWarps);  // one arrival per epilogue warp
    }
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmap_w);
    tma_prefetch_desc(&tmap_x);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, L::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // Grouped mode: the row-block list is written by the previous kernel, so
  // every thread waits for it before reading. Dense mode: the unit list is
  // arithmetic and the producer may request weight tiles before the wait.
  const bool grouped = args.blocks != nullptr;
  if (grouped) pdl_wait();
  const int k_splits = args.k_splits > 1 ? args.k_splits : 1;
  const int k_iters = args.K / kBK / k_splits;  // per split
  const int total_k = args.K / kBK;
  int tiles = total_tiles(args);
  if (tiles < 0 || (args.max_units > 0 && tiles * k_splits > args.max_units)) {
    // a corrupt block count: record it and do no work rather than stream
    // from wild coordinates
    if (threadIdx.x == 0) report_status(args.status, kBoundsViolation, 40);
    tiles = 0;
  }
  const int units = tiles * k_splits;
  // stream-K (grouped, no split-K): only when every CTA's range is at least
  // one tile long, so that a tile has at most two pieces (same on every CTA)
  const bool stream_k = args.stream_k && grouped && k_splits == 1 && tiles > 0 &&
                        (long long)tiles * total_k / gridDim.x >= total_k;

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      // Dense mode: weight tiles are static, so the first unit's weight tiles
      // are requested before waiting on the previous kernel; only the
      // activation tiles wait.
      int pre = 0;
      if (!grouped && (int)blockIdx.x < units) {
        const Unit un = unit_of(blockIdx.x, tiles);
        const int4 blk = unit_block(args, un.tile / args.f_tiles);
        const int n_boxes = (blk.y + kBoxRows - 1) / kBoxRows;
        const int w_row = blk.z * args.w_rows_per_group + (un.tile % args.f_tiles) * kBM;
        const uint32_t bytes = L::kABytes * (SWIGLU ? 2 : 1) + n_boxes * kBoxRows * kBK * 2;
        pre = min(STAGES, k_iters);
        for (int i = 0; i < pre; ++i) {  // fresh stages: nothing to wait for
          uint8_t* sa = smem + i * L::kStageBytes;
          const int k = un.split * k_iters + i;
          mbar_arrive_expect_tx(&full_bar[i], bytes);
          tma_load_2d(sa, &tmap_w, &full_bar[i], k * kBK, w_row);
          if (SWIGLU)
            tma_load_2d(sa + L::kABytes, &tmap_w, &full_bar[i], k * kBK, w_row + args.up_offset);
        }
      }
      pdl_wait();
      pdl_trigger();
      SegIter it(stream_k, tiles, total_k, k_splits);
      int tile_i, k0, k1, piece, pieces;
      while (!*abort_flag && it.next(tile_i, k0, k1, piece, pieces)) {
        const int4 blk = unit_block(args, tile_i / args.f_tiles);
        const int ft = tile_i % args.f_tiles;
        const int n_boxes = (blk.y + kBoxRows - 1) / kBoxRows;
        const int w_row = blk.z * args.w_rows_per_group + ft * kBM;
        const uint32_t bytes = L::kABytes * (SWIGLU ? 2 : 1) + n_boxes * kBoxRows * kBK * 2;
        if (args.row_ids != nullptr) {
          // source rows of this block; padding rows repeat the last real row
          for (int j = 0; j < n_boxes * kBoxRows; ++j)
            rows_s[j] = args.row_ids[blk.x + min(j, blk.y - 1)];
        }
        for (int k = k0; k < k1; ++k) {
          uint8_t* sa = smem + stage * L::kStageBytes;
          uint8_t* sb = sa + L::kABytes * (SWIGLU ? 2 : 1);
          if (pre > 0) {
            --pre;  // weight tile already requested; add the activation boxes
          } else {
            if (!mbar_wait(&empty_bar[stage], phase ^ 1, abort_flag, args.status, 10)) break;
            mbar_arrive_expect_tx(&full_bar[stage], bytes);
            tma_load_2d(sa, &tmap_w, &full_bar[stage], k * kBK, w_row);
            if (SWIGLU)
              tma_load_2d(sa + L::kABytes, &tmap_w, &full_bar[stage], k * kBK,
                          w_row + args.up_offset);
          }
          if (args.row_ids != nullptr) {
            for (int j = 0; j < n_boxes * kBoxRows; j += 4)
              tma_gather4(sb + j * kBK * 2, &tmap_x, &full_bar[stage], k * kBK, rows_s[j],
                          rows_s[j + 1], rows_s[j + 2], rows_s[j + 3]);
          } else {
            for (int b = 0; b < n_boxes; ++b)
              tma_load_2d(sb + b * kBoxRows * kBK * 2, &tmap_x, &full_bar[stage], k * kBK,
                          blk.x + b * kBoxRows);
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      // Drain: the last STAGES fills must have landed before the CTA may
      // exit (their full barriers complete on TMA arrival, independent of
      // the MMA warp). Fills that never happened refer to phases before the
      // barrier's first one and complete immediately.
      volatile int no_abort = 0;
      for (int s = 0; s < STAGES; ++s) {
        if (--stage < 0) { stage = STAGES - 1; phase ^= 1; }
        mbar_wait(&full_bar[stage], phase, &no_abort, args.status, 11);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------- MMA issuer
    pdl_wait();
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      int t = 0;  // local tile counter
      SegIter it(stream_k, tiles, total_k, k_splits);
      int tile_i, k0, k1, piece, pieces;
      for (; !*abort_flag && it.next(tile_i, k0, k1, piece, pieces); ++t) {
        const int4 blk = unit_block(args, tile_i / args.f_tiles);
        const int n_mma = max(32, ((blk.y + 31) / 32) * 32);
        const uint32_t idesc = umma_idesc_bf16(kBM, n_mma);
        const int slot = t % L::kSlots;
        const uint32_t tpar = (uint32_t)((t / L::kSlots) & 1);
        // the epilogue must have drained this slot's previous accumulator
        if (!mbar_wait(&tempty_bar[slot], tpar ^ 1, abort_flag, args.status, 20)) break;
        tc_fence_after();
        const uint32_t d_gate = tmem_base + slot * L::kSlotCols;
        bool ok = true;
        for (int k = k0; k < k1; ++k) {
          if (!mbar_wait(&full_bar[stage], phase, abort_flag, args.status, 21)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * L::kStageBytes);
          const uint32_t sb = sa + L::kABytes * (SWIGLU ? 2 : 1);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint64_t bdesc = umma_desc_sw128(sb + kk * 32);
            const uint32_t acc = (k != k0 || kk != 0) ? 1u : 0u;
            umma_bf16(d_gate, umma_desc_sw128(sa + kk * 32), bdesc, idesc, acc);
            if (SWIGLU)
              umma_bf16(d_gate + L::kAccCols, umma_desc_sw128(sa + L::kABytes + kk * 32), bdesc,
                        idesc, acc);
          }
          umma_commit(&empty_bar[stage]);  // smem stage free once these MMAs retire
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        umma_commit(&tfull_bar[slot]);  // accumulator ready for the epilogue
      }
    }
  } else {
    // --------------------------------------------------------- epilogue
    // TMEM lane quarter q holds features q*32..q*32+31 of the tile. Each
    // 16-column chunk is rounded to bf16 in registers, transposed through a
    // warp-private smem tile [16 rows][32 features], and written as 16-byte
    // row vectors (4 lanes per row), with the residual read the same way.
    pdl_wait();  // residual / row scale / outputs belong to earlier kernels
    const int q = warp & 3;
    __nv_bfloat16* st = stage_out + (warp - 2) * 16 * 32;
    float* sc = scale_s + (warp - 2) * BN;  // this warp's copy of the tile's row scales
    volatile int* last_flag = abort_flag + 1;
    int t = 0;
    SegIter it(stream_k, tiles, total_k, k_splits);
    int tile_i, k0, k1, piece, pieces;
    for (; !*abort_flag && it.next(tile_i, k0, k1, piece, pieces); ++t) {
      const Unit un = {tile_i, piece};
      const int4 blk = unit_block(args, un.tile / args.f_tiles);
      const int ft = un.tile % args.f_tiles;
      const int slot = t % L::kSlots;
      const uint32_t tpar = (uint32_t)((t / L::kSlots) & 1);
      if (!SWIGLU && args.row_scale != nullptr) {
        // the tile's row scales, requested while its MMAs still run
        for (int r = lane; r < blk.y; r += 32) sc[r] = args.row_scale[blk.x + r];
        __syncwarp();
      }
      // warp-uniform: the TMEM loads below are warp-collective
      if (!__all_sync(0xffffffffu, mbar_wait(&tfull_bar[slot], tpar, abort_flag, args.status, 30)))
        break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + ((uint32_t)(q * 32) << 16) + slot * L::kSlotCols;
      const int f_base = ft * kBM + q * 32;
      bool emit = true;
      float* wsp = nullptr;
      if (pieces > 1) {
        // split-K / stream-K piece: store this piece's partial tile (SwiGLU:
        // gate and up) into its own fp32 slice; the last piece to finish sums
        // the slices in piece order, so the result does not depend on which
        // piece finished first
        const size_t tile_elems = (size_t)BN * kBM * (SWIGLU ? 2 : 1);
        wsp = args.ws + (size_t)un.tile * tile_elems + q * 32 + lane;
        float* own = wsp + (size_t)un.split * tiles * tile_elems;
        for (int c = 0; c < blk.y; c += 16) {
          float acc[16];
          tmem_ld16(t_row + c, acc);
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (c + j < blk.y) __stcg(own + (c + j) * kBM, acc[j]);
          if constexpr (SWIGLU) {
            tmem_ld16(t_row + L::kAccCols + c, acc);
#pragma unroll
            for (int j = 0; j < 16; ++j)
              if (c + j < blk.y) __stcg(own + (size_t)BN * kBM + (c + j) * kBM, acc[j]);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty_bar[slot]);  // TMEM slot free already
        __threadfence();
        epi_bar();
        if (threadIdx.x == 64)
          *last_flag = (atomicAdd(&args.tile_counters[un.tile], 1) == pieces - 1);
        epi_bar();
        emit = *last_flag != 0;
        if (emit) __threadfence();
      }
      // 32 accumulator columns (rows of the output) per TMEM load, handled as
      // two 16-row halves through the staging tile
      for (int c0 = 0; c0 < blk.y && emit; c0 += 32) {
      float a32[32], u32[32];
      if (wsp == nullptr) {
        tmem_ld32(t_row + c0, a32);
        if constexpr (SWIGLU) tmem_ld32(t_row + L::kAccCols + c0, u32);
      }
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int c = c0 + 16 * hh;
        if (c >= blk.y) break;
        float acc[16];
        float up[16];
        if (wsp != nullptr) {
          // last split: sum the partial slices in split order; four slices'
          // 16 values are loaded before any is added, so 64 loads are in
          // flight instead of one dependent load at a time
          const size_t split_stride = (size_t)tiles * BN * kBM * (SWIGLU ? 2 : 1);
          auto reduce = [&](float (&out)[16], const float* src) {
#pragma unroll
            for (int j = 0; j < 16; ++j) out[j] = 0.f;
            for (int sp0 = 0; sp0 < pieces; sp0 += 4) {
              float v[4][16];
#pragma unroll
              for (int u = 0; u < 4; ++u)
#pragma unroll
                for (int j = 0; j < 16; ++j)
                  v[u][j] = (sp0 + u < pieces && c + j < blk.y)
                                ? __ldcg(src + (sp0 + u) * split_stride + (c + j) * kBM)
                                : 0.f;
#pragma unroll
              for (int u = 0; u < 4; ++u)
#pragma unroll
                for (int j = 0; j < 16; ++j) out[j] += v[u][j];
            }
          };
          reduce(acc, wsp);
          if constexpr (SWIGLU) reduce(up, wsp + (size_t)BN * kBM);
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) acc[j] = a32[16 * hh + j];
          if constexpr (SWIGLU) {
#pragma unroll
            for (int j = 0; j < 16; ++j) up[j] = u32[16 * hh + j];
          }
        }
        if (SWIGLU) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            // HF rounds gate/up to bf16 before the activation and the product
            const float g = round_bf16(acc[j]);
            const float s = g / (1.0f + __expf(-g));
            acc[j] = round_bf16(s) * round_bf16(up[j]);
          }
        } else if (args.row_scale != nullptr) {
#pragma unroll
          for (int j = 0; j < 16; ++j) acc[j] = round_bf16(acc[j]) * sc[min(c + j, blk.y - 1)];
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) st[j * 32 + lane] = f_to_bf16(acc[j]);
        __syncwarp();
        const int g8 = (lane & 3) * 8;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int j = (lane >> 2) + 8 * h;
          if (c + j < blk.y) {
            const int row = blk.x + c + j;
            uint4 v = *reinterpret_cast<const uint4*>(st + j * 32 + g8);
            const int col = f_base + g8;
            if (args.residual != nullptr) {
              const uint4 r = *reinterpret_cast<const uint4*>(
                  args.residual + (size_t)row * args.ld_res + col);
              const uint32_t* pv = &v.x;
              const uint32_t* pr = &r.x;
              uint32_t o[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                float a0, a1, b0, b1;
                unpack_bf16x2(pv[e], a0, a1);
                unpack_bf16x2(pr[e], b0, b1);
                o[e] = pack_bf16x2(a0 + b0, a1 + b1);
              }
              v = make_uint4(o[0], o[1], o[2], o[3]);
            }
            *reinterpret_cast<uint4*>(args.out + (size_t)row * args.ld_out + col) = v;
            if (args.cmb_inv == nullptr)
              for (int p = 0; p < args.n_peers; ++p)
              *reinterpret_cast<uint4*>(
                  args.peer_out[p] + (size_t)(row + args.peer_row_offset) * args.ld_out + col) = v;
          }
        }
        __syncwarp();
      }
      }
      if (wsp != nullptr) {
        if (emit && threadIdx.x == 64) args.tile_counters[un.tile] = 0;
        continue;  // TMEM slot was released before the reduction
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty_bar[slot]);
      if (args.cmb_inv != nullptr) {
        // the CTA that stores the last row block of feature tile ft combines it
        __threadfence();
        epi_bar();
        if (threadIdx.x == 64)
          *last_flag = (atomicAdd(&args.cmb_counters[ft], 1) == tiles / args.f_tiles - 1);
        epi_bar();
        if (*last_flag) {
          __threadfence();
          combine_feature_tile(args, ft);
          if (threadIdx.x == 64) args.cmb_counters[ft] = 0;
        }
      }
    }
    // no local rows at all: the combine is residual-only (or zeros)
    if (args.cmb_inv != nullptr && tiles == 0 && !*abort_flag && blockIdx.x < args.f_tiles)
      combine_feature_tile(args, blockIdx.x);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, L::kTmemCols);
  }

  // Fused completion signal: the last CTA to finish publishes the flag value
  // to every peer flag (and the local one), after a system-scope fence that
  // orders this CTA's peer stores before its counter increment. An aborted
  // CTA never signals: the consumer's bounded wait then reports the failure
  // instead of reading a half-written tile.
  if (args.done_counter != nullptr && threadIdx.x == 0 && !*abort_flag) {
    fence_sys();
    const int prev = atomicAdd(args.done_counter, 1);
    if (prev == (int)gridDim.x - 1) {
      fence_sys();
      const int v = args.signal_value + (args.epoch != nullptr ? *args.epoch : 0);
      for (int p = 0; p < args.n_flags; ++p) st_release_sys(args.flags[p], v);
      *args.done_counter = 0;
    }
  }
}

// ============================================================ host side ===

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || p == nullptr) return nullptr;
    fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 2-D bf16 row-major [rows, cols] (row stride `ld` elements), box
// {64 cols, box_rows rows}, 128-byte swizzle, zero fill out of bounds.
static int make_tmap(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int64_t ld,
                     int box_rows) {
  EncodeTiledFn enc = get_encode_fn();
  if (enc == nullptr) return -1;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : (int)r;
}

template <bool SWIGLU, int BN, int STAGES>
static cudaError_t launch_variant(const CUtensorMap& tw, const CUtensorMap& tx, const GemmArgs& a,
                                  int grid, cudaStream_t stream) {
  using L = GemmSmem<SWIGLU, BN, STAGES>;
  auto kern = gemm_swapab_kernel<SWIGLU, BN, STAGES>;
  const cudaError_t e = set_max_dynamic_smem(reinterpret_cast<const void*>(kern), L::kTotal);
  if (e != cudaSuccess) return e;
  return launch_k(kern, dim3(grid), dim3(kThreads), L::kTotal, stream, tw, tx, a);
}

int gemm_swapab_launch(const GemmLaunch& p, cudaStream_t stream) {
  if (p.token_major && gemm_tm_eligible(p)) return gemm_tm_launch(p, stream);
  if (p.args.K % kBK != 0) return 1001;
  if (p.w_rows_total <= 0) return 1002;
  if (p.block_n != 64 && p.block_n != 128 && p.block_n != 256) return 1003;
  if (((uintptr_t)p.w & 15) || ((uintptr_t)p.x & 15)) return 1004;
  if (p.args.f_tiles <= 0) return 1005;
  CUtensorMap tw, tx;
  int r = make_tmap(&tw, p.w, p.w_rows_total, p.args.K, p.ld_w, kBM);
  if (r) return 2000 + r;
  // gathered rows: one-row boxes for tile::gather4
  r = make_tmap(&tx, p.x, p.x_rows, p.args.K, p.ld_x, p.args.row_ids != nullptr ? 1 : kBoxRows);
  if (r) return 3000 + r;
  GemmArgs a = p.args;
  a.block_n = p.block_n;
  if (a.stream_k && (a.ws == nullptr || a.tile_counters == nullptr)) return 1009;
  if (a.k_splits > 1) {
    if ((p.args.K / kBK) % a.k_splits != 0) return 1007;
    if (a.ws == nullptr || a.tile_counters == nullptr) return 1008;
  }
  int units_hint = p.units_hint > 0 ? p.units_hint : p.num_sms;
  a.max_units = p.units_hint > 0 ? p.units_hint : 0;
  int grid = units_hint < p.num_sms ? units_hint : p.num_sms;
  if (grid < 1) grid = 1;
  cudaError_t e;
  // stage counts fill ~192 KB of shared memory per CTA (one CTA per SM)
  if (p.swiglu) {
    if (p.block_n == 64) e = launch_variant<true, 64, 5>(tw, tx, a, grid, stream);
    else if (p.block_n == 128) e = launch_variant<true, 128, 4>(tw, tx, a, grid, stream);
    else e = launch_variant<true, 256, 3>(tw, tx, a, grid, stream);
  } else {
    if (p.block_n == 64) e = launch_variant<false, 64, 8>(tw, tx, a, grid, stream);
    else if (p.block_n == 128) e = launch_variant<false, 128, 6>(tw, tx, a, grid, stream);
    else e = launch_variant<false, 256, 4>(tw, tx, a, grid, stream);
  }
  return e == cudaSuccess ? 0 : 4000 + (int)e;
}

}  // namespace afd
