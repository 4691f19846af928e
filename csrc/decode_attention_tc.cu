// GQA decode attention (one query token per sequence) on the 5th-generation
// tensor cores, reading the KV cache with TMA.
//
// For a (sequence, kv head) the G = nq / nkv query heads share K and V, so
// one 128-key tile is two small GEMMs with the keys on the 128 TMEM lanes:
//
//   S^T [128 keys x 16]  = K_tile [128 x 128 dims] . Q^T [128 dims x 16 heads]
//   PV^T [128 dims x 16] = V_tile^T [128 dims x 128 keys] . P^T [128 keys x 16]
//
// (heads G..15 are padding: the MMA's N is 16). K is the K-major A operand of
// the first product straight from its TMA tile; V is the MN-major A operand
// of the second, also straight from its tile, so nothing is transposed. Both
// accumulators live in TMEM, double buffered by tile, so the S product of
// tile i+1 and the PV product of tile i overlap the softmax. The online
// softmax runs on 4 warps, one key per thread: each tile's per-head maximum
// is exchanged through shared memory at a named barrier of the 4 warps, P^T
// is written to shared memory in the 128-byte-swizzled K-major layout, and
// the output O (one head-dim lane per thread, G heads) is rescaled in
// registers, so TMEM is never written back.
//
// Work items are (sequence, kv head, key split); a persistent grid of at
// most one CTA per SM walks them, so the TMA producer streams the next
// item's tiles while the softmax warps finish the current one. With more
// than one split, each item writes fp32 partials (O, running max, sum) and
// the last split of a (sequence, kv head) to finish merges them with all 128
// softmax threads (a per-pair counter that the merging CTA resets), so one
// launch computes the result.
//
//   warp 0      TMA producer: Q (16 rows) per item, K/V 128-key tiles into a
//               3-stage ring
//   warp 1      TMEM owner and MMA issuer (one elected lane)
//   warps 2..5  softmax, output, split merge
//
// Fused new-token step (qkv given): the softmax warps apply the q RMSNorm and
// RoPE to the token's query heads and write Q^T straight into shared memory
// (no TMA for Q), and the CTA whose split owns the tile holding the new
// position first normalises/ropes the token's key and appends K and V to the
// cache; the producer issues that tile's TMA only after those stores, made
// visible to the async proxy. One kernel per layer then covers what a
// norm/RoPE/append kernel plus an attention kernel would.
//
// The position of the query token, *start_pos, is read on the device (a
// captured CUDA graph replays as the cache grows). A position outside
// [0, s_max) reads no key, writes zeros and records kBoundsViolation.
// head_dim 128; every wait is bounded (mbar_wait) and unwinds on timeout.
//
// No cluster launch and no multicast: every TMA load reads this GPU's memory.

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "common.cuh"
#include "kernels.h"

namespace afd {

namespace {

constexpr int kDD = 128;                       // head dim
constexpr int kDKeys = 128;                    // keys per tile (TMEM lanes)
constexpr int kDN = 16;                        // MMA N: query heads, padded
constexpr int kDBox = kDKeys * 128;            // one SW128 box: 128 rows x 64 bf16 (16 KB)
constexpr int kDTile = 2 * kDBox;              // a 128 x 128 K or V tile (32 KB)
constexpr int kDStages = 3;
constexpr int kDQBytes = kDN * kDD * 2;        // 4 KB: two boxes of 16 rows x 128 B
constexpr int kDPBytes = kDN * kDKeys * 2;     // 4 KB: two 64-key atoms of 16 rows
constexpr int kDThreads = 192;
constexpr uint32_t kDTmemCols = 64;            // S[2] and PV[2], 16 columns each
constexpr int kDMaxSplits = 64;                // key splits per (sequence, kv head)
constexpr int kDSmem = kDStages * 2 * kDTile + 2 * kDQBytes + 2 * kDPBytes + 1024 /*align*/ +
                       1024 /*barriers + exchange*/ + 8 * kDMaxSplits * 2 * 4 /*merge*/;

__device__ __forceinline__ void item_of(const DecodeTcArgs& a, int w, int& b, int& kvh,
                                        int& split) {
  split = w % a.nsplit;
  kvh = (w / a.nsplit) % a.nkv;
  b = w / (a.nsplit * a.nkv);
}

// Key-tile range [t0, t1) of split `split` when the sequence has n_tiles.
__device__ __forceinline__ void split_range(int n_tiles, int nsplit, int split, int& t0,
                                            int& t1) {
  const int per = (n_tiles + nsplit - 1) / nsplit;
  t0 = min(n_tiles, split * per);
  t1 = min(n_tiles, t0 + per);
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Byte offset of P^T[head h][key r] in the K-major, 128-byte-swizzled B
// operand: two 64-key atoms of 16 rows x 128 B (8-row groups 1024 B apart).
__device__ __forceinline__ uint32_t p_offset(int h, int r) {
  const int j = r >> 6, kk = r & 63;
  return j * 2048 + (h >> 3) * 1024 + (h & 7) * 128 + ((((kk >> 3) ^ (h & 7))) << 4) +
         (kk & 7) * 2;
}

// Byte offset of Q^T[head h][dim d] in the K-major, 128-byte-swizzled B
// operand of the S product: two 64-dim boxes of 16 rows x 128 B.
__device__ __forceinline__ uint32_t q_offset(int h, int d) {
  const int c = d & 63;
  return (d >> 6) * 2048 + (h >> 3) * 1024 + (h & 7) * 128 + ((((c >> 3) ^ (h & 7))) << 4) +
         (c & 7) * 2;
}

// RMSNorm over the 128 dims of one head row, then RoPE at `pos`, HF roundings
// (bf16 after the norm, the weight, each RoPE product and the sum). Lane l
// owns dims 2l, 2l+1 (y[0], y[1]) and their rotation partners 64+2l, 65+2l
// (y[2], y[3]).
__device__ __forceinline__ void norm_rope_lane(const __nv_bfloat16* src, const __nv_bfloat16* nw,
                                               const float* rope, int pos, float eps, int lane,
                                               float (&y)[4]) {
  const int j = 2 * lane;
  float x[4];
  unpack_bf16x2(*reinterpret_cast<const uint32_t*>(src + j), x[0], x[1]);
  unpack_bf16x2(*reinterpret_cast<const uint32_t*>(src + 64 + j), x[2], x[3]);
  float w[4];
  unpack_bf16x2(*reinterpret_cast<const uint32_t*>(nw + j), w[0], w[1]);
  unpack_bf16x2(*reinterpret_cast<const uint32_t*>(nw + 64 + j), w[2], w[3]);
  float ss = x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float rstd = rsqrtf(ss / 128.f + eps);
  const float2 c = *reinterpret_cast<const float2*>(rope + (size_t)pos * 128 + j);
  const float2 sn = *reinterpret_cast<const float2*>(rope + (size_t)pos * 128 + 64 + j);
  const float cv[2] = {c.x, c.y}, sv[2] = {sn.x, sn.y};
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const float xl = round_bf16(w[e] * round_bf16(x[e] * rstd));
    const float xh = round_bf16(w[2 + e] * round_bf16(x[2 + e] * rstd));
    y[e] = round_bf16(round_bf16(xl * cv[e]) + round_bf16(-xh * sv[e]));
    y[2 + e] = round_bf16(round_bf16(xh * cv[e]) + round_bf16(xl * sv[e]));
  }
}

// Instruction descriptor with an MN-major A operand (bit 15) on top of the
// common kind::f16 fields.
__device__ __forceinline__ uint32_t idesc_a_mn(int M, int N) {
  return umma_idesc_bf16(M, N) | (1u << 15);
}

}  // namespace

template <int G>
__global__ void __launch_bounds__(kDThreads, 1)
    decode_attention_tc_kernel(const __grid_constant__ CUtensorMap tq,
                               const __grid_constant__ CUtensorMap tk,
                               const __grid_constant__ CUtensorMap tv, DecodeTcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* kv_s = smem;                                   // stage s: K at 2s, V at 2s+1
  uint8_t* q_s = kv_s + kDStages * 2 * kDTile;            // [2] items
  uint8_t* p_s = q_s + 2 * kDQBytes;                      // [2] tiles
  uint64_t* bars = reinterpret_cast<uint64_t*>(p_s + 2 * kDPBytes);
  uint64_t* kv_full = bars;                               // [kDStages]
  uint64_t* kv_empty = bars + kDStages;                   // [kDStages]
  uint64_t* q_full = bars + 2 * kDStages;                 // [2]
  uint64_t* q_empty = q_full + 2;                         // [2]
  uint64_t* s_full = q_empty + 2;                         // [2]
  uint64_t* s_free = s_full + 2;                          // [2]
  uint64_t* p_full = s_free + 2;                          // [2]
  uint64_t* pv_full = p_full + 2;                         // [2]
  uint64_t* pv_free = pv_full + 2;                        // [2]
  uint64_t* kv_new = pv_free + 2;                         // new token's K/V stored (fused)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(kv_new + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* merge_flag = abort_flag + 1;
  float* red = reinterpret_cast<float*>(tmem_slot + 8);   // [2][4 warps][16] tile maxima
  float* sred = red + 2 * 4 * kDN;                        // [4 warps][16] sums, then merge area

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const bool fused = a.qkv != nullptr;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kDStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], fused ? 4 : 1);  // softmax warps write Q, or one TMA
      mbar_init(&q_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 4);
      mbar_init(&p_full[i], 4);
      mbar_init(&pv_full[i], 1);
      mbar_init(&pv_free[i], 4);
    }
    mbar_init(kv_new, 4);
    *abort_flag = 0;
    fence_barrier_init();
    if (!fused) tma_prefetch_desc(&tq);
    tma_prefetch_desc(&tk);
    tma_prefetch_desc(&tv);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kDTmemCols);
    tmem_relinquish();
  }
  // the padding rows G..15 of both P^T buffers stay zero
  for (int i = threadIdx.x; i < 2 * kDPBytes / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(p_s)[i] = make_uint4(0, 0, 0, 0);
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  pdl_wait();  // q and the cache rows come from the previous kernels
  pdl_trigger();
  int kv_len = *a.start_pos + 1;
  if (kv_len < 1 || kv_len > a.s_max) {
    if (threadIdx.x == 0 && blockIdx.x == 0) report_status(a.status, kBoundsViolation, 62);
    kv_len = 0;
  }
  const int n_tiles = (kv_len + kDKeys - 1) / kDKeys;
  const int n_items = a.B * a.nkv * a.nsplit;

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer
    if (elect_one()) {
      int g = 0, qi = 0;
      for (int w = blockIdx.x; w < n_items && !*abort_flag; w += gridDim.x) {
        int b, kvh, split, t0, t1;
        item_of(a, w, b, kvh, split);
        split_range(n_tiles, a.nsplit, split, t0, t1);
        if (t1 <= t0) continue;
        if (!fused) {
          const int qb = qi & 1;
          if (qi >= 2 &&
              !mbar_wait(&q_empty[qb], ((qi >> 1) - 1) & 1, abort_flag, a.status, 80))
            break;
          mbar_arrive_expect_tx(&q_full[qb], kDQBytes);
          for (int c = 0; c < 2; ++c)
            tma_load_2d(q_s + qb * kDQBytes + c * (kDQBytes / 2), &tq, &q_full[qb], c * 64,
                        b * a.nq + kvh * G);
        }
        ++qi;
        const int plane = (a.batch_offset + b) * a.nkv + kvh;
        bool ok = true;
        for (int t = t0; t < t1; ++t, ++g) {
          const int st = g % kDStages;
          if (g >= kDStages &&
              !mbar_wait(&kv_empty[st], ((g / kDStages) - 1) & 1, abort_flag, a.status, 81)) {
            ok = false;
            break;
          }
          if (fused && t == n_tiles - 1 && !mbar_wait(kv_new, 0, abort_flag, a.status, 89)) {
            // this tile holds the new position: its K/V rows must be stored first
            ok = false;
            break;
          }
          uint8_t* ks = kv_s + (2 * st) * kDTile;
          uint8_t* vs = ks + kDTile;
          mbar_arrive_expect_tx(&kv_full[st], 2 * kDTile);
          for (int c = 0; c < 2; ++c) {
            tma_load_3d(ks + c * kDBox, &tk, &kv_full[st], c * 64, t * kDKeys, plane);
            tma_load_3d(vs + c * kDBox, &tv, &kv_full[st], c * 64, t * kDKeys, plane);
          }
        }
        if (!ok) break;
      }
      // Drain: the loads in flight must land before the CTA exits.
      volatile int no_abort = 0;
      for (int x = max(0, g - kDStages); x < g; ++x)
        mbar_wait(&kv_full[x % kDStages], (x / kDStages) & 1, &no_abort, nullptr, 82,
                  100000000ull);
      if (!fused)
        for (int x = max(0, qi - 2); x < qi; ++x)
          mbar_wait(&q_full[x & 1], (x >> 1) & 1, &no_abort, nullptr, 83, 100000000ull);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------- MMA issuer
    if (elect_one()) {
      const uint32_t idesc_s = umma_idesc_bf16(kDKeys, kDN);
      const uint32_t idesc_pv = idesc_a_mn(kDD, kDN);
      const uint32_t pa = smem_u32(p_s);
      int g = 0, qi = 0;
      int prev = -1;  // global index of the tile whose PV product is pending
      bool ok = true;
      auto issue_pv = [&](int x) -> bool {
        const int pb = x & 1;
        if (!mbar_wait(&p_full[pb], (x >> 1) & 1, abort_flag, a.status, 84)) return false;
        if (x >= 2 && !mbar_wait(&pv_free[pb], ((x >> 1) - 1) & 1, abort_flag, a.status, 85))
          return false;
        tc_fence_after();
        const uint32_t va = smem_u32(kv_s + (2 * (x % kDStages) + 1) * kDTile);
#pragma unroll
        for (int kk = 0; kk < kDKeys / 16; ++kk) {
          // 16 keys = two 8-row groups of the V tile; the 128 dims span its two boxes
          const uint64_t ad = umma_desc_sw128_mn(va + kk * 2048, kDBox, 1024);
          const uint64_t bd =
              umma_desc_sw128(pa + pb * kDPBytes + (kk >> 2) * 2048 + (kk & 3) * 32);
          umma_bf16(tmem + 32 + pb * kDN, ad, bd, idesc_pv, kk > 0 ? 1u : 0u);
        }
        umma_commit(&pv_full[pb]);
        umma_commit(&kv_empty[x % kDStages]);
        return true;
      };
      for (int w = blockIdx.x; ok && w < n_items && !*abort_flag; w += gridDim.x) {
        int b, kvh, split, t0, t1;
        item_of(a, w, b, kvh, split);
        split_range(n_tiles, a.nsplit, split, t0, t1);
        if (t1 <= t0) continue;
        // The previous item's last PV product first: in the fused step the
        // softmax warps write this item's Q only after consuming it.
        if (prev >= 0) {
          if (!issue_pv(prev)) {
            ok = false;
            break;
          }
          prev = -1;
        }
        const int qb = qi & 1;
        if (!mbar_wait(&q_full[qb], (qi >> 1) & 1, abort_flag, a.status, 86)) break;
        const uint32_t qa = smem_u32(q_s + qb * kDQBytes);
        for (int t = t0; t < t1; ++t, ++g) {
          const int st = g % kDStages, sb = g & 1;
          if (!mbar_wait(&kv_full[st], (g / kDStages) & 1, abort_flag, a.status, 87) ||
              (g >= 2 && !mbar_wait(&s_free[sb], ((g >> 1) - 1) & 1, abort_flag, a.status, 88))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t ka = smem_u32(kv_s + (2 * st) * kDTile);
#pragma unroll
          for (int kk = 0; kk < kDD / 16; ++kk) {
            const uint32_t off = (kk >> 2) * kDBox + (kk & 3) * 32;
            const uint32_t qoff = (kk >> 2) * (kDQBytes / 2) + (kk & 3) * 32;
            umma_bf16(tmem + sb * kDN, umma_desc_sw128(ka + off), umma_desc_sw128(qa + qoff),
                      idesc_s, kk > 0 ? 1u : 0u);
          }
          umma_commit(&s_full[sb]);
          if (t == t1 - 1) umma_commit(&q_empty[qb]);  // Q buffer free once these retire
          if (prev >= 0 && !issue_pv(prev)) {
            ok = false;
            break;
          }
          prev = g;
        }
        ++qi;
      }
      if (ok && prev >= 0) issue_pv(prev);
    }
  } else {
    // -------------------------------------------------- softmax + output
    // The 4 softmax warps meet at named barrier 1 (128 threads) in a fixed
    // sequence: once per tile (the per-head tile maximum), once per item (the
    // per-head sums) and, with splits, twice per item (partials written; the
    // merge decision) plus twice per merge. A warp whose bounded wait failed
    // keeps walking the same sequence without touching TMEM or memory, so no
    // warp is left waiting at a barrier; after an abort every wait returns at
    // once.
    const int qq = warp & 3;               // TMEM lane quarter of this warp
    const int r = qq * 32 + lane;          // key row of a tile / head-dim lane of O
    const uint32_t lane_off = (uint32_t)(qq * 32) << 16;
    const float scale = rsqrtf((float)kDD) * 1.4426950408889634f;  // log2 domain
    const int pos = kv_len - 1;
    if (fused) {
      // The new token's K (normed + roped) and V of every item of this CTA
      // whose split owns the last tile, before the producer loads that tile:
      // (item, k or v) pairs spread over the 4 warps. Stores, then a proxy
      // fence so the TMA (async proxy) sees them, then one arrival per warp.
      int job = 0;
      for (int w = blockIdx.x; w < n_items && kv_len > 0; w += gridDim.x) {
        int b, kvh, split, t0, t1;
        item_of(a, w, b, kvh, split);
        split_range(n_tiles, a.nsplit, split, t0, t1);
        if (!(t0 <= n_tiles - 1 && n_tiles - 1 < t1)) continue;
        const __nv_bfloat16* row = a.qkv + (size_t)b * a.ld_qkv;
        const size_t crow = (((size_t)(a.batch_offset + b) * a.nkv + kvh) * a.s_max + pos) * kDD;
        for (int which = 0; which < 2; ++which, ++job) {
          if (job % 4 != qq) continue;
          if (which == 0) {
            float y[4];
            norm_rope_lane(row + (size_t)(a.nq + kvh) * kDD, a.k_norm, a.rope, pos, a.eps, lane,
                           y);
            __nv_bfloat16* dst = a.k_cache + crow;
            *reinterpret_cast<uint32_t*>(dst + 2 * lane) = pack_bf16x2(y[0], y[1]);
            *reinterpret_cast<uint32_t*>(dst + 64 + 2 * lane) = pack_bf16x2(y[2], y[3]);
          } else {
            const uint2 v = *reinterpret_cast<const uint2*>(
                row + (size_t)(a.nq + a.nkv + kvh) * kDD + 4 * lane);
            *reinterpret_cast<uint2*>(a.v_cache + crow + 4 * lane) = v;
          }
        }
      }
      fence_proxy_async_global();
      __syncwarp();
      if (lane == 0) mbar_arrive(kv_new);
    }
    // wait for an mbarrier phase with the whole warp; false (and `ok` cleared)
    // on timeout or abort
    bool ok = true;
    auto wait_all = [&](uint64_t* bar, uint32_t parity, int where) -> bool {
      if (ok && !__all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag, a.status, where)))
        ok = false;
      return ok;
    };
    int g = 0, qi = 0;
    for (int w = blockIdx.x; w < n_items; w += gridDim.x) {
      int b, kvh, split, t0, t1;
      item_of(a, w, b, kvh, split);
      split_range(n_tiles, a.nsplit, split, t0, t1);
      if (fused && t1 > t0) {
        // Q^T of this item: RMSNorm + RoPE of its G query heads into the
        // shared-memory operand (warp qq takes heads qq, qq + 4, ...)
        const int qb = qi & 1;
        if (qi < 2 || wait_all(&q_empty[qb], ((qi >> 1) - 1) & 1, 97)) {
          uint8_t* qs = q_s + qb * kDQBytes;
          const __nv_bfloat16* row = a.qkv + (size_t)b * a.ld_qkv;
          for (int h = qq; h < G; h += 4) {
            float y[4];
            norm_rope_lane(row + (size_t)(kvh * G + h) * kDD, a.q_norm, a.rope, pos, a.eps,
                           lane, y);
            *reinterpret_cast<uint32_t*>(qs + q_offset(h, 2 * lane)) = pack_bf16x2(y[0], y[1]);
            *reinterpret_cast<uint32_t*>(qs + q_offset(h, 64 + 2 * lane)) =
                pack_bf16x2(y[2], y[3]);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&q_full[qb]);
        }
      }
      if (t1 > t0) ++qi;
      float m_run[G], l_part[G], o[G], alpha_prev[G];
#pragma unroll
      for (int h = 0; h < G; ++h) {
        m_run[h] = -INFINITY;
        l_part[h] = 0.f;
        o[h] = 0.f;
        alpha_prev[h] = 0.f;
      }
      for (int t = t0; t < t1; ++t, ++g) {
        const int sb = g & 1;
        float s[16];
        if (wait_all(&s_full[sb], (g >> 1) & 1, 90)) {
          tc_fence_after();
          tmem_ld16(tmem + lane_off + sb * kDN, s);
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&s_free[sb]);
        }
        const int key = t * kDKeys + r;
        const bool valid = ok && key < kv_len;
        float x[G];
#pragma unroll
        for (int h = 0; h < G; ++h) {
          x[h] = valid ? s[h] * scale : -INFINITY;
          const float wm = warp_max(x[h]);
          if (lane == h) red[(sb * 4 + qq) * kDN + h] = wm;
        }
        named_bar_sync(1, 128);
        float alpha[G], p[G];
#pragma unroll
        for (int h = 0; h < G; ++h) {
          float tm = red[(sb * 4 + 0) * kDN + h];
          tm = fmaxf(tm, red[(sb * 4 + 1) * kDN + h]);
          tm = fmaxf(tm, red[(sb * 4 + 2) * kDN + h]);
          tm = fmaxf(tm, red[(sb * 4 + 3) * kDN + h]);
          // finite on a healthy path (every tile holds a valid key); after a
          // failure nothing below is stored
          const float m_new = fmaxf(m_run[h], tm);
          alpha[h] = m_new == -INFINITY ? 0.f : exp2f(m_run[h] - m_new);  // 0 on the first tile
          m_run[h] = m_new;
          p[h] = valid ? exp2f(x[h] - m_new) : 0.f;
          l_part[h] = l_part[h] * alpha[h] + p[h];
        }
        if (ok && t == n_tiles - 1 && t * kDKeys + kDKeys > kv_len &&
            wait_all(&kv_full[g % kDStages], (g / kDStages) & 1, 92) && key >= kv_len) {
          // rows past the sequence end in the last tile: zero V so that
          // P = 0 meets finite values in the PV product
          uint8_t* vs = kv_s + (2 * (g % kDStages) + 1) * kDTile;
#pragma unroll
          for (int c = 0; c < 2; ++c)
#pragma unroll
            for (int u = 0; u < 8; ++u)
              *reinterpret_cast<uint4*>(vs + c * kDBox + r * 128 + u * 16) = make_uint4(0, 0, 0, 0);
        }
        if (ok) {
          // P^T into this tile's buffer (the PV product two tiles back, which
          // read it, completed before its PV was consumed)
          uint8_t* pb_s = p_s + sb * kDPBytes;
#pragma unroll
          for (int h = 0; h < G; ++h)
            *reinterpret_cast<__nv_bfloat16*>(pb_s + p_offset(h, r)) = f_to_bf16(p[h]);
          fence_proxy_async_smem();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&p_full[sb]);
        }
        if (t > t0 && wait_all(&pv_full[(g - 1) & 1], ((g - 1) >> 1) & 1, 93)) {
          // O += the previous tile's PV, after rescaling O to its max
          const int xb = (g - 1) & 1;
          tc_fence_after();
          float pv[16];
          tmem_ld16(tmem + lane_off + 32 + xb * kDN, pv);
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&pv_free[xb]);
#pragma unroll
          for (int h = 0; h < G; ++h) o[h] = o[h] * alpha_prev[h] + pv[h];
        }
#pragma unroll
        for (int h = 0; h < G; ++h) alpha_prev[h] = alpha[h];
      }
      float l[G];
#pragma unroll
      for (int h = 0; h < G; ++h) l[h] = 0.f;
      if (t1 > t0) {
        if (wait_all(&pv_full[(g - 1) & 1], ((g - 1) >> 1) & 1, 94)) {
          const int xb = (g - 1) & 1;
          tc_fence_after();
          float pv[16];
          tmem_ld16(tmem + lane_off + 32 + xb * kDN, pv);
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&pv_free[xb]);
#pragma unroll
          for (int h = 0; h < G; ++h) o[h] = o[h] * alpha_prev[h] + pv[h];
        }
        // per-head sums over the 128 key lanes
#pragma unroll
        for (int h = 0; h < G; ++h) {
          const float ws = warp_sum_f(l_part[h]);
          if (lane == h) sred[qq * kDN + h] = ws;
        }
        named_bar_sync(1, 128);
#pragma unroll
        for (int h = 0; h < G; ++h)
          l[h] = sred[0 * kDN + h] + sred[1 * kDN + h] + sred[2 * kDN + h] + sred[3 * kDN + h];
        // sred is rewritten at the next item's end, after its per-tile
        // barriers, which every warp passes only after these reads
      }
      const size_t hq0 = (size_t)b * a.nq + kvh * G;
      if (a.nsplit == 1) {
        if (ok) {
#pragma unroll
          for (int h = 0; h < G; ++h)
            a.out[(hq0 + h) * kDD + r] = f_to_bf16(l[h] > 0.f ? o[h] / l[h] : 0.f);
        }
        continue;
      }
      // split partials (running max in natural-log units); the last split of
      // the (sequence, kv head) to finish merges them, all 128 threads
      if (ok) {
#pragma unroll
        for (int h = 0; h < G; ++h) {
          a.o_part[((hq0 + h) * a.nsplit + split) * kDD + r] = o[h];
          if (r == 0) {
            a.ml_part[((hq0 + h) * a.nsplit + split) * 2 + 0] =
                m_run[h] == -INFINITY ? -INFINITY : m_run[h] * 0.6931471805599453f;
            a.ml_part[((hq0 + h) * a.nsplit + split) * 2 + 1] = l[h];
          }
        }
      }
      __threadfence();
      named_bar_sync(1, 128);
      if (threadIdx.x == 64)
        *merge_flag = ok && !*abort_flag &&
                      atomicAdd(&a.counters[b * a.nkv + kvh], 1) == a.nsplit - 1;
      named_bar_sync(1, 128);
      const bool merge = *merge_flag != 0;
      // merge_flag is rewritten only after the next item's barriers
      if (merge) {
        __threadfence();
        // (max, sum) of every split of every head into shared memory first
        // (one batch of loads), then thread r sums its head-dim lane
        float* ml_s = sred + 4 * kDN;  // [G][nsplit][2], nsplit <= kDMaxSplits
        for (int i = r; i < G * a.nsplit * 2; i += 128)
          ml_s[i] = __ldcg(a.ml_part + hq0 * a.nsplit * 2 + i);
        named_bar_sync(1, 128);
#pragma unroll
        for (int h = 0; h < G; ++h) {
          const float* mh = ml_s + h * a.nsplit * 2;
          float M = -INFINITY;
          for (int sp = 0; sp < a.nsplit; ++sp) M = fmaxf(M, mh[2 * sp]);
          float L = 0.f, acc = 0.f;
          const float* op = a.o_part + (hq0 + h) * a.nsplit * kDD + r;
#pragma unroll 4
          for (int sp = 0; sp < a.nsplit; ++sp) {
            const float ms = mh[2 * sp];
            const float wgt = ms == -INFINITY ? 0.f : __expf(ms - M);
            L += mh[2 * sp + 1] * wgt;
            acc += __ldcg(op + (size_t)sp * kDD) * wgt;
          }
          a.out[(hq0 + h) * kDD + r] = f_to_bf16(L > 0.f ? acc / L : 0.f);
        }
        if (threadIdx.x == 64) a.counters[b * a.nkv + kvh] = 0;
        named_bar_sync(1, 128);  // ml_s is reused by the next merge
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kDTmemCols);
  }
}

// ============================================================ host side ===

typedef CUresult (*EncodeTiledFnDec)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                     const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                     const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                     CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFnDec dec_encode_fn() {
  static EncodeTiledFnDec fn = nullptr;
  if (fn == nullptr) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || p == nullptr) return nullptr;
    fn = reinterpret_cast<EncodeTiledFnDec>(p);
  }
  return fn;
}

static int dec_encode(CUtensorMap* m, const void* base, int rank, const cuuint64_t* dims,
                      const cuuint64_t* strides, const cuuint32_t* box) {
  EncodeTiledFnDec enc = dec_encode_fn();
  if (enc == nullptr) return -1;
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(base), dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : 100 + (int)r;
}

int decode_tc_supported(int nq, int nkv, int D) {
  if (D != kDD || nkv <= 0 || nq % nkv != 0) return 0;
  const int G = nq / nkv;
  return G == 8 || G == 4;
}

int launch_decode_attention_tc(const DecodeTcArgs& a, int grid, cudaStream_t s) {
  if (!decode_tc_supported(a.nq, a.nkv, a.D) || a.nsplit < 1 || a.nsplit > kDMaxSplits || a.B < 0)
    return 1;
  if (a.nsplit > 1 && (a.o_part == nullptr || a.ml_part == nullptr || a.counters == nullptr))
    return 2;
  if ((a.qkv == nullptr && (a.q == nullptr || ((uintptr_t)a.q & 15))) ||
      ((uintptr_t)a.k_cache & 15) || ((uintptr_t)a.v_cache & 15))
    return 3;
  if (a.qkv != nullptr && (((uintptr_t)a.qkv & 7) || (a.ld_qkv & 3) || a.q_norm == nullptr ||
                           a.k_norm == nullptr || a.rope == nullptr))
    return 3;
  if (a.B == 0) return 0;
  CUtensorMap tq, tk, tv;
  memset(&tq, 0, sizeof(tq));
  if (a.qkv == nullptr) {  // q [B * nq, 128]: 16 rows per box (a kv head's G heads + padding)
    cuuint64_t dims[2] = {(cuuint64_t)kDD, (cuuint64_t)a.B * a.nq};
    cuuint64_t str[1] = {(cuuint64_t)kDD * 2};
    cuuint32_t box[2] = {64, (cuuint32_t)kDN};
    int e = dec_encode(&tq, a.q, 2, dims, str, box);
    if (e) return e;
  }
  const cuuint64_t planes = (cuuint64_t)(a.batch_offset + a.B) * a.nkv;
  cuuint64_t kdims[3] = {(cuuint64_t)kDD, (cuuint64_t)a.s_max, planes};
  cuuint64_t kstr[2] = {(cuuint64_t)kDD * 2, (cuuint64_t)a.s_max * kDD * 2};
  cuuint32_t kbox[3] = {64, (cuuint32_t)kDKeys, 1};
  int e = dec_encode(&tk, a.k_cache, 3, kdims, kstr, kbox);
  if (e) return e;
  e = dec_encode(&tv, a.v_cache, 3, kdims, kstr, kbox);
  if (e) return e;
  const int G = a.nq / a.nkv;
  const int items = a.B * a.nkv * a.nsplit;
  const int g = grid < items ? grid : items;
  cudaError_t r;
  if (G == 8) {
    r = set_max_dynamic_smem(reinterpret_cast<const void*>(decode_attention_tc_kernel<8>), kDSmem);
    if (r == cudaSuccess)
      r = launch_k(decode_attention_tc_kernel<8>, dim3(g), dim3(kDThreads), kDSmem, s, tq, tk, tv,
                   a);
  } else {
    r = set_max_dynamic_smem(reinterpret_cast<const void*>(decode_attention_tc_kernel<4>), kDSmem);
    if (r == cudaSuccess)
      r = launch_k(decode_attention_tc_kernel<4>, dim3(g), dim3(kDThreads), kDSmem, s, tq, tk, tv,
                   a);
  }
  return r == cudaSuccess ? 0 : 4000 + (int)r;
}

}  // namespace afd
