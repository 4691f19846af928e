// Token-major grouped GEMM on the 5th-generation tensor cores, for
// prefill-sized batches:
//
//   out[row, f] = epilogue( sum_k X[row, k] * W[group, f, k] )
//
// The token rows are the MMA's A operand (M = 128 rows of one row block) and
// the weights the B operand (N = 256: 256 output features, or for SwiGLU 128
// gate rows and the matching 128 up rows), so the accumulator has one token
// row per TMEM lane and the features along the columns. Against the swap-AB
// kernel (gemm_tcgen05.cu, weights as A, N = the block's token count), each
// MMA is 128 x 256 instead of 128 x 128, which reads 12 KB of shared memory
// per 128 x 256 x 16 product instead of 16 KB for the same work as two
// 128 x 128 products, and the epilogue writes each thread's own output row
// segment straight to global memory (64-byte runs) with no transpose through
// shared memory. Decode-sized batches (a few rows per expert) stay on the
// swap-AB kernel, where N follows the row count.
//
// Work units are (row block, feature tile) as in the swap-AB kernel, from the
// MoE routing's block list or a dense row count; a persistent grid deals them
// round-robin. Warp roles (192 threads): warp 0 TMA producer, warp 1 TMEM
// owner + MMA issuer, warps 2..5 epilogue. Two TMEM accumulators of 256
// columns let the MMA warp run one tile ahead of the epilogue. Every wait is
// bounded; a timeout records a status and aborts the CTA.
//
// Supported epilogues: SwiGLU (gate/up pair -> act), per-row scale (routing
// weight), residual add, peer stores and the completion flag. Not here:
// split-K, gathered rows (tile::gather4) and the fused combine; the launcher
// sends those to the swap-AB kernel.
//
// No cluster launch: every TMA load is issued per CTA and reads this GPU's memory.

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "gemm_tcgen05.h"

namespace afd {

namespace {

constexpr int kTmBM = 128;       // token rows per tile (MMA M)
constexpr int kTmN = 256;        // MMA N: weight rows per tile
constexpr int kTmBK = 64;        // K per stage (one 128-byte swizzle atom)
constexpr int kTmStages = 4;
constexpr int kTmThreads = 192;
constexpr int kTmABytes = kTmBM * kTmBK * 2;   // 16 KB
constexpr int kTmBBytes = kTmN * kTmBK * 2;    // 32 KB
constexpr int kTmStageBytes = kTmABytes + kTmBBytes;
constexpr int kTmSmem = kTmStages * kTmStageBytes + 1024 /*align*/ + 256 /*barriers*/;

__device__ __forceinline__ int4 tm_block(const GemmArgs& a, int b) {
  if (a.blocks != nullptr) return a.blocks[b];
  const int rs = b * kTmBM;
  return make_int4(rs, min(kTmBM, a.dense_rows - rs), 0, 0);
}

// 16 fp32 -> 8 packed bf16 pairs
__device__ __forceinline__ void pack16(const float* v, uint32_t* o) {
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
}

}  // namespace

// f_tiles counts output-feature tiles of this kernel: 256 features (plain)
// or 128 (SwiGLU) per tile.
template <bool SWIGLU>
__global__ void __launch_bounds__(kTmThreads, 1)
    gemm_tm_kernel(const __grid_constant__ CUtensorMap tmap_w,
                   const __grid_constant__ CUtensorMap tmap_x, const GemmArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + kTmStages * kTmStageBytes);
  uint64_t* empty_bar = full_bar + kTmStages;
  uint64_t* tfull_bar = empty_bar + kTmStages;   // [2]
  uint64_t* tempty_bar = tfull_bar + 2;          // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty_bar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kTmStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&tfull_bar[s], 1);
      mbar_init(&tempty_bar[s], 4);  // one arrival per epilogue warp
    }
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmap_w);
    tma_prefetch_desc(&tmap_x);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const bool grouped = args.blocks != nullptr;
  if (grouped) pdl_wait();
  const int k_iters = args.K / kTmBK;
  const int nb = grouped ? *args.num_blocks : (args.dense_rows + kTmBM - 1) / kTmBM;
  int tiles = nb * args.f_tiles;
  if (nb < 0 || (args.max_units > 0 && tiles > args.max_units)) {
    if (threadIdx.x == 0) report_status(args.status, kBoundsViolation, 45);
    tiles = 0;
  }
  // weight rows of feature tile ft of group g: plain 256 rows from ft * 256;
  // SwiGLU 128 gate rows from ft * 128 and the 128 up rows up_offset later
  auto w_rows = [&](int g, int ft, int& r0, int& r1) {
    const int base = g * args.w_rows_per_group;
    if (SWIGLU) {
      r0 = base + ft * 128;
      r1 = r0 + args.up_offset;
    } else {
      r0 = base + ft * 256;
      r1 = r0 + 128;
    }
  };

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      // dense mode: the first tile's weight stages are requested before the
      // dependency wait (weights are static); only the token rows wait
      int pre = 0;
      if (!grouped && (int)blockIdx.x < tiles) {
        const int4 blk = tm_block(args, blockIdx.x / args.f_tiles);
        int r0, r1;
        w_rows(blk.z, blockIdx.x % args.f_tiles, r0, r1);
        pre = min(kTmStages, k_iters);
        for (int i = 0; i < pre; ++i) {
          uint8_t* sb = smem + i * kTmStageBytes + kTmABytes;
          mbar_arrive_expect_tx(&full_bar[i], kTmStageBytes);
          tma_load_2d(sb, &tmap_w, &full_bar[i], i * kTmBK, r0);
          tma_load_2d(sb + kTmBBytes / 2, &tmap_w, &full_bar[i], i * kTmBK, r1);
        }
      }
      pdl_wait();
      pdl_trigger();
      for (int t = blockIdx.x; t < tiles && !*abort_flag; t += gridDim.x) {
        const int4 blk = tm_block(args, t / args.f_tiles);
        int r0, r1;
        w_rows(blk.z, t % args.f_tiles, r0, r1);
        for (int k = 0; k < k_iters; ++k) {
          uint8_t* sa = smem + stage * kTmStageBytes;
          uint8_t* sb = sa + kTmABytes;
          if (pre > 0) {
            --pre;  // weights already requested; add the token rows
          } else {
            if (!mbar_wait(&empty_bar[stage], phase ^ 1, abort_flag, args.status, 12)) break;
            mbar_arrive_expect_tx(&full_bar[stage], kTmStageBytes);
            tma_load_2d(sb, &tmap_w, &full_bar[stage], k * kTmBK, r0);
            tma_load_2d(sb + kTmBBytes / 2, &tmap_w, &full_bar[stage], k * kTmBK, r1);
          }
          tma_load_2d(sa, &tmap_x, &full_bar[stage], k * kTmBK, blk.x);
          if (++stage == kTmStages) { stage = 0; phase ^= 1; }
        }
      }
      // every fill must land before the CTA exits
      volatile int no_abort = 0;
      for (int s = 0; s < kTmStages; ++s) {
        if (--stage < 0) { stage = kTmStages - 1; phase ^= 1; }
        mbar_wait(&full_bar[stage], phase, &no_abort, args.status, 13);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------- MMA issuer
    pdl_wait();
    if (elect_one()) {
      const uint32_t idesc = umma_idesc_bf16(kTmBM, kTmN);
      int stage = 0;
      uint32_t phase = 0;
      int n = 0;  // local tile counter
      for (int t = blockIdx.x; t < tiles && !*abort_flag; t += gridDim.x, ++n) {
        const int slot = n & 1;
        if (!mbar_wait(&tempty_bar[slot], ((n >> 1) & 1) ^ 1, abort_flag, args.status, 22)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + slot * kTmN;
        bool ok = true;
        for (int k = 0; k < k_iters; ++k) {
          if (!mbar_wait(&full_bar[stage], phase, abort_flag, args.status, 23)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * kTmStageBytes);
          const uint32_t sb = sa + kTmABytes;
#pragma unroll
          for (int kk = 0; kk < kTmBK / 16; ++kk)
            umma_bf16(d, umma_desc_sw128(sa + kk * 32), umma_desc_sw128(sb + kk * 32), idesc,
                      (k | kk) != 0);
          umma_commit(&empty_bar[stage]);
          if (++stage == kTmStages) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        umma_commit(&tfull_bar[slot]);
      }
    }
  } else {
    // --------------------------------------------------------- epilogue
    // thread = one token row of the tile (TMEM lane q * 32 + lane)
    pdl_wait();  // residual / row scale / outputs belong to earlier kernels
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    constexpr int kOutF = SWIGLU ? 128 : 256;  // output features per tile
    int n = 0;
    for (int t = blockIdx.x; t < tiles && !*abort_flag; t += gridDim.x, ++n) {
      const int4 blk = tm_block(args, t / args.f_tiles);
      const int f0 = (t % args.f_tiles) * kOutF;
      const int slot = n & 1;
      const bool valid = r < blk.y;
      const size_t row = (size_t)blk.x + r;
      float scale = 1.f;
      if (!SWIGLU && args.row_scale != nullptr && valid) scale = args.row_scale[row];
      if (!__all_sync(0xffffffffu,
                      mbar_wait(&tfull_bar[slot], (n >> 1) & 1, abort_flag, args.status, 31)))
        break;
      tc_fence_after();
      const uint32_t t_acc = tmem_base + lane_off + slot * kTmN;
#pragma unroll 1
      for (int c = 0; c < kOutF; c += 32) {
        float v[32];
        tmem_ld32(t_acc + c, v);
        if constexpr (SWIGLU) {
          float u[32];
          tmem_ld32(t_acc + 128 + c, u);
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            // HF rounds gate/up to bf16 before the activation and the product
            const float g = round_bf16(v[j]);
            const float s = g / (1.0f + __expf(-g));
            v[j] = round_bf16(s) * round_bf16(u[j]);
          }
        } else if (args.row_scale != nullptr) {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = round_bf16(v[j]) * scale;
        }
        if (!valid) continue;
        uint32_t o[16];
        if (args.residual != nullptr) {
          // (bf16 result) + residual in fp32, rounded once: the swap-AB epilogue's order
          const uint4* rp =
              reinterpret_cast<const uint4*>(args.residual + row * args.ld_res + f0 + c);
#pragma unroll
          for (int w = 0; w < 4; ++w) {
            const uint4 rv = rp[w];
            const uint32_t* pr = &rv.x;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              float r0, r1;
              unpack_bf16x2(pr[e], r0, r1);
              const int j = w * 8 + 2 * e;
              o[w * 4 + e] = pack_bf16x2(round_bf16(v[j]) + r0, round_bf16(v[j + 1]) + r1);
            }
          }
        } else {
          pack16(v, o);
          pack16(v + 16, o + 8);
        }
        uint4* dst = reinterpret_cast<uint4*>(args.out + row * args.ld_out + f0 + c);
#pragma unroll
        for (int w = 0; w < 4; ++w)
          dst[w] = make_uint4(o[4 * w], o[4 * w + 1], o[4 * w + 2], o[4 * w + 3]);
        for (int p = 0; p < args.n_peers; ++p) {
          uint4* pd = reinterpret_cast<uint4*>(
              args.peer_out[p] + (row + args.peer_row_offset) * args.ld_out + f0 + c);
#pragma unroll
          for (int w = 0; w < 4; ++w)
            pd[w] = make_uint4(o[4 * w], o[4 * w + 1], o[4 * w + 2], o[4 * w + 3]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty_bar[slot]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }

  // the last CTA publishes the completion flag (see gemm_swapab_kernel)
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

typedef CUresult (*EncodeTiledFnTm)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                    const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                    const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                    CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFnTm tm_encode_fn() {
  static EncodeTiledFnTm fn = nullptr;
  if (fn == nullptr) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || p == nullptr) return nullptr;
    fn = reinterpret_cast<EncodeTiledFnTm>(p);
  }
  return fn;
}

// bf16 row-major [rows, cols] (row stride ld), box {64, 128 rows}, SW128
static int tm_tmap(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int64_t ld) {
  EncodeTiledFnTm enc = tm_encode_fn();
  if (enc == nullptr) return -1;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {(cuuint32_t)kTmBK, 128u};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : (int)r;
}

bool gemm_tm_eligible(const GemmLaunch& p) {
  const GemmArgs& a = p.args;
  if (p.block_n != kTmBM || a.k_splits > 1 || a.row_ids != nullptr || a.cmb_inv != nullptr)
    return false;
  if (a.K % kTmBK != 0) return false;
  // f_tiles arrive in 128-feature units: plain tiles take two of them
  if (!p.swiglu && (a.f_tiles % 2 != 0)) return false;
  if (p.swiglu && a.up_offset % 128 != 0) return false;
  // 16-byte row segments in the epilogue
  if ((a.ld_out % 8) != 0 || (a.residual != nullptr && (a.ld_res % 8) != 0)) return false;
  if (((uintptr_t)a.out & 15) || ((uintptr_t)a.residual & 15)) return false;
  for (int i = 0; i < a.n_peers; ++i)
    if ((uintptr_t)a.peer_out[i] & 15) return false;
  return true;
}

int gemm_tm_launch(const GemmLaunch& p, cudaStream_t stream) {
  if (!gemm_tm_eligible(p)) return 1;
  if (((uintptr_t)p.w & 15) || ((uintptr_t)p.x & 15)) return 1004;
  CUtensorMap tw, tx;
  int r = tm_tmap(&tw, p.w, p.w_rows_total, p.args.K, p.ld_w);
  if (r) return 2000 + r;
  r = tm_tmap(&tx, p.x, p.x_rows, p.args.K, p.ld_x);
  if (r) return 3000 + r;
  GemmArgs a = p.args;
  a.block_n = kTmBM;
  if (!p.swiglu) a.f_tiles /= 2;  // 256-feature tiles
  // units bound: the caller's hint is in 128-feature tiles
  a.max_units = p.units_hint > 0 ? p.units_hint : 0;
  int grid = p.num_sms;
  if (p.units_hint > 0 && p.units_hint < grid) grid = p.units_hint;
  if (grid < 1) grid = 1;
  cudaError_t e;
  if (p.swiglu) {
    e = set_max_dynamic_smem(reinterpret_cast<const void*>(gemm_tm_kernel<true>), kTmSmem);
    if (e == cudaSuccess)
      e = launch_k(gemm_tm_kernel<true>, dim3(grid), dim3(kTmThreads), kTmSmem, stream, tw, tx, a);
  } else {
    e = set_max_dynamic_smem(reinterpret_cast<const void*>(gemm_tm_kernel<false>), kTmSmem);
    if (e == cudaSuccess)
      e = launch_k(gemm_tm_kernel<false>, dim3(grid), dim3(kTmThreads), kTmSmem, stream, tw, tx,
                   a);
  }
  return e == cudaSuccess ? 0 : 4000 + (int)e;
}

}  // namespace afd
