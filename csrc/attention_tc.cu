// Causal GQA flash-attention prefill on the 5th-generation tensor cores.
//
// One CTA per (128-query tile, query head, sequence). Q, K and V tiles move
// global -> shared memory with TMA (128-byte swizzle); S = Q K^T and
// O += P V run as tcgen05.mma with both accumulators in TMEM (S: columns
// 0..127, O: columns 128..255, one lane per query row). The online softmax
// reads S from TMEM, writes P (bf16) into shared memory as the K-major A
// operand of the PV product, and rescales O in TMEM when a row's running max
// grows. V is used as an MN-major B operand straight from its TMA tile, so no
// transpose is needed.
//
//   warp 0      TMA producer: Q once, then K/V tiles into a 2-stage ring
//   warp 1      TMEM owner and MMA issuer (one elected lane)
//   warps 2..5  softmax + O rescale + epilogue, one query row per thread
//
// S_{j+1} is issued as soon as the softmax warps have read S_j into
// registers, so it overlaps the softmax of tile j; P_j V_j follows when P_j
// is in shared memory. Every wait is bounded (mbar_wait); a timeout aborts
// the CTA without hanging the GPU.
//
// Same contract as prefill_attention_kernel (attention.cu): q [B*q_len, nq,
// D], caches [B_max, nkv, s_max, D], queries at positions start_pos ..
// start_pos + q_len - 1 (start_pos read on the device) attend to keys
// 0 .. their own position. D = 128.

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "kernels.h"

namespace afd {

namespace {

constexpr int kTcD = 128;          // head dim
constexpr int kTcBM = 128;         // queries per CTA (TMEM lanes)
constexpr int kTcBN = 128;         // keys per tile
constexpr int kTcChunk = 128 * 128;            // one SW128 box: 128 rows x 64 bf16
constexpr int kTcTile = 2 * kTcChunk;          // 128 rows x 128 bf16 (two boxes)
constexpr int kTcStages = 2;
constexpr int kTcThreads = 192;
constexpr int kTcSmem = kTcTile /*Q*/ + kTcStages * 2 * kTcTile /*K,V*/ + kTcTile /*P*/ +
                        1024 /*align*/ + 256 /*barriers*/;
constexpr uint32_t kTmemCols = 256;

struct TcMaps {
  CUtensorMap q, k, v;
};

__device__ __forceinline__ void softmax_bar() {  // the 4 softmax warps
  asm volatile("bar.sync 1, 128;" ::: "memory");
}

}  // namespace

__global__ void __launch_bounds__(kTcThreads, 1)
    prefill_attention_tc_kernel(const __grid_constant__ CUtensorMap tq,
                                const __grid_constant__ CUtensorMap tk,
                                const __grid_constant__ CUtensorMap tv, PrefillAttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* q_s = smem;
  uint8_t* kv_s = q_s + kTcTile;                       // stage s: K at 2s, V at 2s+1
  uint8_t* p_s = kv_s + kTcStages * 2 * kTcTile;
  uint64_t* bars = reinterpret_cast<uint64_t*>(p_s + kTcTile);
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 1;                        // [2]
  uint64_t* kv_empty = bars + 3;                       // [2]
  uint64_t* s_full = bars + 5;
  uint64_t* s_free = bars + 6;
  uint64_t* p_full = bars + 7;
  uint64_t* o_done = bars + 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 9);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int qtile = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int G = a.nq / a.nkv;
  const int kvh = h / G;
  const int q0 = qtile * kTcBM;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kTcStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, 4);
    mbar_init(p_full, 4);
    mbar_init(o_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tq);
    tma_prefetch_desc(&tk);
    tma_prefetch_desc(&tv);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_s = tmem;            // S: columns [0, 128)
  const uint32_t t_o = tmem + kTcBN;    // O: columns [128, 256)

  pdl_wait();
  pdl_trigger();
  const int start = *a.start_pos;
  const int kv_len = start + a.q_len;
  // keys any row of this tile can see: 0 .. start + q0 + 127 (and < kv_len)
  const int last_key = min(kv_len, start + q0 + kTcBM) - 1;
  const int n_tiles = q0 < a.q_len ? last_key / kTcBN + 1 : 0;
  const int kv_plane = (a.batch_offset + b) * a.nkv + kvh;

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer
    if (elect_one() && n_tiles > 0) {
      mbar_arrive_expect_tx(q_full, kTcTile);
      for (int c = 0; c < 2; ++c) tma_load_4d(q_s + c * kTcChunk, &tq, q_full, c * 64, h, q0, b);
      int issued = 0;
      for (int j = 0; j < n_tiles && !*abort_flag; ++j) {
        const int st = j % kTcStages;
        if (j >= kTcStages &&
            !mbar_wait(&kv_empty[st], ((j / kTcStages) - 1) & 1, abort_flag, nullptr, 60))
          break;
        ++issued;
        uint8_t* ks = kv_s + (2 * st) * kTcTile;
        uint8_t* vs = ks + kTcTile;
        mbar_arrive_expect_tx(&kv_full[st], 2 * kTcTile);
        for (int c = 0; c < 2; ++c) {
          tma_load_3d(ks + c * kTcChunk, &tk, &kv_full[st], c * 64, j * kTcBN, kv_plane);
          tma_load_3d(vs + c * kTcChunk, &tv, &kv_full[st], c * 64, j * kTcBN, kv_plane);
        }
      }
      // Drain: every load issued must land before the CTA exits (normally
      // the MMA warp has consumed them all already; after an abort it has not)
      volatile int no_abort = 0;
      mbar_wait(q_full, 0, &no_abort, nullptr, 66, 100000000ull);
      for (int j = max(0, issued - kTcStages); j < issued; ++j)
        mbar_wait(&kv_full[j % kTcStages], (j / kTcStages) & 1, &no_abort, nullptr, 67,
                  100000000ull);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------- MMA issuer
    if (elect_one() && n_tiles > 0) {
      const uint32_t idesc_s = umma_idesc_bf16(kTcBM, kTcBN);
      const uint32_t idesc_pv = umma_idesc_bf16(kTcBM, kTcD, /*b_mn_major=*/true);
      const uint32_t qa = smem_u32(q_s), pa = smem_u32(p_s);
      auto issue_s = [&](int j) {
        const uint32_t ka = smem_u32(kv_s + (2 * (j % kTcStages)) * kTcTile);
#pragma unroll
        for (int kk = 0; kk < kTcD / 16; ++kk) {
          const uint32_t off = (kk / 4) * kTcChunk + (kk % 4) * 32;
          umma_bf16(t_s, umma_desc_sw128(qa + off), umma_desc_sw128(ka + off), idesc_s, kk > 0);
        }
        umma_commit(s_full);
      };
      bool ok = mbar_wait(q_full, 0, abort_flag, nullptr, 61) &&
                mbar_wait(&kv_full[0], 0, abort_flag, nullptr, 62);
      if (ok) {
        tc_fence_after();
        issue_s(0);
      }
      for (int j = 0; ok && j < n_tiles; ++j) {
        if (j + 1 < n_tiles) {
          // S_{j+1} as soon as the softmax holds S_j in registers
          const int sn = (j + 1) % kTcStages;
          if (!mbar_wait(&kv_full[sn], ((j + 1) / kTcStages) & 1, abort_flag, nullptr, 63) ||
              !mbar_wait(s_free, j & 1, abort_flag, nullptr, 64))
            break;
          tc_fence_after();
          issue_s(j + 1);
        }
        if (!mbar_wait(p_full, j & 1, abort_flag, nullptr, 65)) break;
        tc_fence_after();
        const uint32_t va = smem_u32(kv_s + (2 * (j % kTcStages) + 1) * kTcTile);
#pragma unroll
        for (int kk = 0; kk < kTcBN / 16; ++kk) {
          const uint64_t ad = umma_desc_sw128(pa + (kk / 4) * kTcChunk + (kk % 4) * 32);
          // 16 keys = two 8-row groups of the V tile; D spans its two 64-wide boxes
          const uint64_t bd = umma_desc_sw128_mn(va + kk * 2048, kTcChunk, 1024);
          umma_bf16(t_o, ad, bd, idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(o_done);
        umma_commit(&kv_empty[j % kTcStages]);
      }
    }
  } else {
    // ------------------------------------------- softmax + O correction
    const int qq = warp & 3;              // TMEM lane quarter of this warp
    const int row = qq * 32 + lane;
    const int pos = start + q0 + row;     // this query's position
    const uint32_t lane_off = (uint32_t)(qq * 32) << 16;
    const float scale = rsqrtf((float)kTcD);
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    // TMEM loads/stores are warp-collective (.sync.aligned): every branch
    // around them is taken by the whole warp (warp-uniform predicates), or
    // the warp would wait for lanes that never arrive.
    for (int j = 0; j < n_tiles; ++j) {
      if (!__all_sync(0xffffffffu, mbar_wait(s_full, j & 1, abort_flag, nullptr, 70))) {
        ok = false;
        break;
      }
      tc_fence_after();
      float s[kTcBN];
#pragma unroll
      for (int c = 0; c < kTcBN / 16; ++c) {
        float t[16];
        tmem_ld16(t_s + lane_off + c * 16, t);
#pragma unroll
        for (int i = 0; i < 16; ++i) s[c * 16 + i] = t[i];
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_free);
      const int key0 = j * kTcBN;
      float rmax = -INFINITY;
#pragma unroll
      for (int i = 0; i < kTcBN; ++i) {
        const int key = key0 + i;
        s[i] = (key <= pos && key < kv_len) ? s[i] * scale : -INFINITY;
        rmax = fmaxf(rmax, s[i]);
      }
      const float m_new = fmaxf(m, rmax);
      if (j > 0) {
        // P_{j-1} V_{j-1} must be done before O is rescaled or P overwritten
        if (!__all_sync(0xffffffffu, mbar_wait(o_done, (j - 1) & 1, abort_flag, nullptr, 71))) {
          ok = false;
          break;
        }
        tc_fence_after();
        // rows whose max grew scale O by alpha; the others by 1 (same warp pass)
        const bool grow = m_new > m;
        if (__any_sync(0xffffffffu, grow)) {
          const float alpha = grow ? __expf(m - m_new) : 1.f;
          l *= alpha;
#pragma unroll
          for (int c = 0; c < kTcD / 16; ++c) {
            float o[16];
            tmem_ld16(t_o + lane_off + c * 16, o);
#pragma unroll
            for (int i = 0; i < 16; ++i) o[i] *= alpha;
            tmem_st16(t_o + lane_off + c * 16, o);
          }
          tmem_wait_st();
        }
      }
      m = m_new;
      float psum = 0.f;
#pragma unroll
      for (int i = 0; i < kTcBN; ++i) {
        s[i] = s[i] == -INFINITY ? 0.f : __expf(s[i] - m);
        psum += s[i];
      }
      l += psum;
      // P row -> shared memory, K-major with the 128-byte swizzle
#pragma unroll
      for (int u = 0; u < kTcBN / 8; ++u) {
        uint4 v;
        v.x = pack_bf16x2(s[u * 8 + 0], s[u * 8 + 1]);
        v.y = pack_bf16x2(s[u * 8 + 2], s[u * 8 + 3]);
        v.z = pack_bf16x2(s[u * 8 + 4], s[u * 8 + 5]);
        v.w = pack_bf16x2(s[u * 8 + 6], s[u * 8 + 7]);
        const int chunk = u / 8, uc = u % 8;
        *reinterpret_cast<uint4*>(p_s + chunk * kTcChunk + row * 128 + ((uc ^ (row & 7)) * 16)) =
            v;
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    const bool done = ok && n_tiles > 0 &&
                      __all_sync(0xffffffffu, mbar_wait(o_done, (n_tiles - 1) & 1, abort_flag,
                                                        nullptr, 72));
    if (done) {
      tc_fence_after();
      const float inv = 1.f / l;
      const bool valid = q0 + row < a.q_len;
      __nv_bfloat16* dst = a.out + (((size_t)b * a.q_len + q0 + row) * a.nq + h) * kTcD;
#pragma unroll
      for (int c = 0; c < kTcD / 16; ++c) {
        float o[16];
        tmem_ld16(t_o + lane_off + c * 16, o);
        if (valid) {
          uint4 v0, v1;
          v0.x = pack_bf16x2(o[0] * inv, o[1] * inv);
          v0.y = pack_bf16x2(o[2] * inv, o[3] * inv);
          v0.z = pack_bf16x2(o[4] * inv, o[5] * inv);
          v0.w = pack_bf16x2(o[6] * inv, o[7] * inv);
          v1.x = pack_bf16x2(o[8] * inv, o[9] * inv);
          v1.y = pack_bf16x2(o[10] * inv, o[11] * inv);
          v1.z = pack_bf16x2(o[12] * inv, o[13] * inv);
          v1.w = pack_bf16x2(o[14] * inv, o[15] * inv);
          *reinterpret_cast<uint4*>(dst + c * 16) = v0;
          *reinterpret_cast<uint4*>(dst + c * 16 + 8) = v1;
        }
      }
    }
    softmax_bar();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ------------------------------------------------------------------------
// Two query heads per CTA (ping-pong). The two heads of one GQA group share
// every K/V tile, and their softmax warpgroups alternate with the tensor
// core: while warpgroup A turns S_A into P_A, the MMA warp runs P_B V and
// S_B of the next tile, and the other way round. P stays in TMEM: the
// softmax stores it as packed bf16 over the first 64 columns of its own S
// accumulator and the PV product reads it from there as the A operand
// (tcgen05.mma with A in tensor memory), so shared memory holds only Q and
// the K/V ring. Two MMAs into different accumulators are not ordered by
// issue, so S_X(j+1), which overwrites P_X(j), is issued only once
// P_X(j) V_j has completed (a commit barrier per head); a commit tracks
// every earlier MMA of the thread, so "S_X(j+1) complete" also means
// "O_X holds P_X(j) V_j" and the softmax may rescale O_X.
//
// The running max is raised lazily: a row rescales O and its sum only when
// its max grows by more than 8 (log2 units, i.e. a factor 256), otherwise
// P is taken against the older, smaller max (values up to 256, exact in the
// final O / l). This is the conditional rescaling of FlashAttention-4.
//
//   warp 0      TMA producer: both Q tiles once, then K/V tiles (2-stage ring)
//   warp 1      TMEM owner (512 columns) and MMA issuer
//   warps 2..5  softmax of head A, warps 6..9 softmax of head B
//
// TMEM columns: S_A/P_A [0,128), S_B/P_B [128,256), O_A [256,384),
// O_B [384,512). Grid: one CTA per (query tile, head pair, sequence), the
// query tiles with the most keys first.

namespace {

constexpr int kP2Threads = 320;
constexpr int kP2Smem = 2 * kTcTile /*Q_A, Q_B*/ + kTcStages * 2 * kTcTile /*K,V*/ +
                        1024 /*align*/ + 256 /*barriers*/;

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 32 lanes x 32 bit, 16 consecutive columns per thread, raw 32-bit words.
__device__ __forceinline__ void tmem_st16_u32(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32"
      " [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};"
      ::"r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]),
        "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]),
        "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

// D (TMEM) (+)= A (TMEM, K-major, 128 lanes x 16 bf16) x B (shared memory).
__device__ __forceinline__ void umma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

}  // namespace

__global__ void __launch_bounds__(kP2Threads, 1)
    prefill_attention_tc2_kernel(const __grid_constant__ CUtensorMap tq,
                                 const __grid_constant__ CUtensorMap tk,
                                 const __grid_constant__ CUtensorMap tv, PrefillAttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* q_s = smem;                                 // head X at X * kTcTile
  uint8_t* kv_s = q_s + 2 * kTcTile;                   // stage s: K at 2s, V at 2s+1
  uint64_t* bars = reinterpret_cast<uint64_t*>(kv_s + kTcStages * 2 * kTcTile);
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 1;                        // [2]
  uint64_t* kv_empty = bars + 3;                       // [2]
  uint64_t* s_full = bars + 5;                         // [2] per head
  uint64_t* p_full = bars + 7;                         // [2] per head
  uint64_t* o_done = bars + 9;                         // [2] per head
  uint64_t* pv_done = bars + 11;                       // [2] per head
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 13);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int n_qt = (a.q_len + kTcBM - 1) / kTcBM;
  const int pairs = a.nq / 2;
  const int per_qt = (int)gridDim.x / n_qt;          // head pairs x sequences
  // heaviest query tiles (most key tiles) first
  const int qtile = n_qt - 1 - (int)blockIdx.x / per_qt;
  const int rest = (int)blockIdx.x % per_qt;
  const int h0 = 2 * (rest % pairs), b = rest / pairs;
  const int G = a.nq / a.nkv;
  const int kvh = h0 / G;
  const int q0 = qtile * kTcBM;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kTcStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(&s_full[x], 1);
      mbar_init(&p_full[x], 4);
      mbar_init(&o_done[x], 1);
      mbar_init(&pv_done[x], 1);
    }
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tq);
    tma_prefetch_desc(&tk);
    tma_prefetch_desc(&tv);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  pdl_wait();
  pdl_trigger();
  const int start = *a.start_pos;
  const int kv_len = start + a.q_len;
  const int last_key = min(kv_len, start + q0 + kTcBM) - 1;
  const int n_tiles = q0 < a.q_len ? last_key / kTcBN + 1 : 0;
  const int kv_plane = (a.batch_offset + b) * a.nkv + kvh;

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer
    if (elect_one() && n_tiles > 0) {
      mbar_arrive_expect_tx(q_full, 2 * kTcTile);
      for (int x = 0; x < 2; ++x)
        for (int c = 0; c < 2; ++c)
          tma_load_4d(q_s + x * kTcTile + c * kTcChunk, &tq, q_full, c * 64, h0 + x, q0, b);
      int issued = 0;
      for (int j = 0; j < n_tiles && !*abort_flag; ++j) {
        const int st = j % kTcStages;
        if (j >= kTcStages &&
            !mbar_wait(&kv_empty[st], ((j / kTcStages) - 1) & 1, abort_flag, nullptr, 80))
          break;
        ++issued;
        uint8_t* ks = kv_s + (2 * st) * kTcTile;
        uint8_t* vs = ks + kTcTile;
        mbar_arrive_expect_tx(&kv_full[st], 2 * kTcTile);
        for (int c = 0; c < 2; ++c) {
          tma_load_3d(ks + c * kTcChunk, &tk, &kv_full[st], c * 64, j * kTcBN, kv_plane);
          tma_load_3d(vs + c * kTcChunk, &tv, &kv_full[st], c * 64, j * kTcBN, kv_plane);
        }
      }
      // every load issued must land before the CTA exits
      volatile int no_abort = 0;
      mbar_wait(q_full, 0, &no_abort, nullptr, 86, 100000000ull);
      for (int j = max(0, issued - kTcStages); j < issued; ++j)
        mbar_wait(&kv_full[j % kTcStages], (j / kTcStages) & 1, &no_abort, nullptr, 87,
                  100000000ull);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------- MMA issuer
    if (elect_one() && n_tiles > 0) {
      const uint32_t idesc_s = umma_idesc_bf16(kTcBM, kTcBN);
      const uint32_t idesc_pv = umma_idesc_bf16(kTcBM, kTcD, /*b_mn_major=*/true);
      const uint32_t q_base = smem_u32(q_s), kv_base = smem_u32(kv_s);
      auto issue_s = [=](int x, int j) {
        const uint32_t qa = q_base + x * kTcTile;
        const uint32_t ka = kv_base + (2 * (j % kTcStages)) * kTcTile;
#pragma unroll
        for (int kk = 0; kk < kTcD / 16; ++kk) {
          const uint32_t off = (kk / 4) * kTcChunk + (kk % 4) * 32;
          umma_bf16(tmem + x * kTcBN, umma_desc_sw128(qa + off), umma_desc_sw128(ka + off),
                    idesc_s, kk > 0);
        }
        umma_commit(&s_full[x]);
      };
      bool ok = mbar_wait(q_full, 0, abort_flag, nullptr, 81) &&
                mbar_wait(&kv_full[0], 0, abort_flag, nullptr, 82);
      if (ok) {
        tc_fence_after();
        issue_s(0, 0);
        issue_s(1, 0);
      }
      for (int j = 0; ok && j < n_tiles; ++j) {
        const uint32_t va = smem_u32(kv_s + (2 * (j % kTcStages) + 1) * kTcTile);
        for (int x = 0; x < 2 && ok; ++x) {
          if (!mbar_wait(&p_full[x], j & 1, abort_flag, nullptr, 83)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t t_p = tmem + x * kTcBN, t_o = tmem + 2 * kTcBN + x * kTcD;
#pragma unroll
          for (int kk = 0; kk < kTcBN / 16; ++kk) {
            // 16 keys: 8 TMEM columns of packed P; two 8-row groups of the V tile
            const uint64_t bd = umma_desc_sw128_mn(va + kk * 2048, kTcChunk, 1024);
            umma_bf16_ts(t_o, t_p + kk * 8, bd, idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&pv_done[x]);
          if (x == 1) umma_commit(&kv_empty[j % kTcStages]);  // K_j and V_j fully used
          if (j + 1 < n_tiles) {
            if (x == 0 && !mbar_wait(&kv_full[(j + 1) % kTcStages], ((j + 1) / kTcStages) & 1,
                                     abort_flag, nullptr, 84)) {
              ok = false;
              break;
            }
            // S_X(j+1) overwrites P_X(j): only after P_X(j) V_j has read it
            if (!mbar_wait(&pv_done[x], j & 1, abort_flag, nullptr, 85)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_s(x, j + 1);
          } else {
            umma_commit(&o_done[x]);
          }
        }
      }
    }
  } else {
    // ------------------------------------------- softmax + O correction
    const int x = (warp - 2) / 4;         // head of this warpgroup
    const int qq = warp & 3;              // TMEM lane quarter of this warp
    const int row = qq * 32 + lane;
    const int pos = start + q0 + row;
    const int warp_pos0 = start + q0 + qq * 32;  // the position of this warp's first row
    const uint32_t lane_off = (uint32_t)(qq * 32) << 16;
    const uint32_t t_s = tmem + x * kTcBN, t_o = tmem + 2 * kTcBN + x * kTcD;
    const float scale_log2 = rsqrtf((float)kTcD) * 1.4426950408889634f;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    // TMEM loads/stores are warp-collective: every branch around them is
    // warp-uniform
    for (int j = 0; j < n_tiles; ++j) {
      if (!__all_sync(0xffffffffu, mbar_wait(&s_full[x], j & 1, abort_flag, nullptr, 90))) {
        ok = false;
        break;
      }
      tc_fence_after();
      float s[kTcBN];
      tmem_ld128(t_s + lane_off, s);  // four loads, one wait
      const int key0 = j * kTcBN;
      float rmax = -INFINITY;
      // warp-uniform: every key of the tile is visible to every row of this
      // warp (the tile lies below the diagonal and inside the sequence)
      if (key0 + kTcBN - 1 <= warp_pos0 && key0 + kTcBN <= kv_len) {
#pragma unroll
        for (int i = 0; i < kTcBN; ++i) rmax = fmaxf(rmax, s[i]);
      } else {
#pragma unroll
        for (int i = 0; i < kTcBN; ++i) {
          const int key = key0 + i;
          if (key > pos || key >= kv_len) s[i] = -INFINITY;
          rmax = fmaxf(rmax, s[i]);
        }
      }
      rmax *= scale_log2;  // the max in log2 units (m is kept in these)
      // lazy max: move it only when it grows by more than 8 (log2 units)
      const bool grow = rmax > m + 8.f;
      const float m_new = grow ? rmax : m;
      // S_X(j) complete => P_X(j-1) V_{j-1} complete: O_X may be rescaled
      if (j > 0 && __any_sync(0xffffffffu, grow)) {
        const float alpha = grow ? ex2_approx(m - m_new) : 1.f;
        l *= alpha;
#pragma unroll
        for (int c = 0; c < kTcD / 16; ++c) {
          float o[16];
          tmem_ld16(t_o + lane_off + c * 16, o);
#pragma unroll
          for (int i = 0; i < 16; ++i) o[i] *= alpha;
          tmem_st16(t_o + lane_off + c * 16, o);
        }
      }
      m = m_new;
      // p = 2^(s * scale * log2(e) - m); a masked s = -inf gives 2^-inf = 0
      // (m is finite: key 0 is visible to every row in tile 0)
      const float neg_m = -m;
      float psum = 0.f;
#pragma unroll
      for (int c = 0; c < kTcBN / 32; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float p0 = ex2_approx(fmaf(s[c * 32 + 2 * i], scale_log2, neg_m));
          const float p1 = ex2_approx(fmaf(s[c * 32 + 2 * i + 1], scale_log2, neg_m));
          psum += p0 + p1;
          pk[i] = pack_bf16x2(p0, p1);
        }
        // P_X(j), keys c*32 .. c*32+31, over S_X's columns c*16 .. c*16+15
        tmem_st16_u32(t_s + lane_off + c * 16, pk);
      }
      l += psum;
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[x]);
    }
    const bool done = ok && n_tiles > 0 &&
                      __all_sync(0xffffffffu, mbar_wait(&o_done[x], 0, abort_flag, nullptr, 91));
    if (done) {
      tc_fence_after();
      const float inv = 1.f / l;
      const bool valid = q0 + row < a.q_len;
      __nv_bfloat16* dst = a.out + (((size_t)b * a.q_len + q0 + row) * a.nq + h0 + x) * kTcD;
#pragma unroll
      for (int c = 0; c < kTcD / 16; ++c) {
        float o[16];
        tmem_ld16(t_o + lane_off + c * 16, o);
        if (valid) {
          uint4 v0, v1;
          v0.x = pack_bf16x2(o[0] * inv, o[1] * inv);
          v0.y = pack_bf16x2(o[2] * inv, o[3] * inv);
          v0.z = pack_bf16x2(o[4] * inv, o[5] * inv);
          v0.w = pack_bf16x2(o[6] * inv, o[7] * inv);
          v1.x = pack_bf16x2(o[8] * inv, o[9] * inv);
          v1.y = pack_bf16x2(o[10] * inv, o[11] * inv);
          v1.z = pack_bf16x2(o[12] * inv, o[13] * inv);
          v1.w = pack_bf16x2(o[14] * inv, o[15] * inv);
          *reinterpret_cast<uint4*>(dst + c * 16) = v0;
          *reinterpret_cast<uint4*>(dst + c * 16 + 8) = v1;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ============================================================ host side ===

typedef CUresult (*EncodeTiledFnTc)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                    const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                    const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                    CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFnTc encode_fn() {
  static EncodeTiledFnTc fn = nullptr;
  if (fn == nullptr) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || p == nullptr) return nullptr;
    fn = reinterpret_cast<EncodeTiledFnTc>(p);
  }
  return fn;
}

// bf16 tensor of `rank` dims (dims[0] innermost, byte strides of dims 1..),
// box {64, box[1], ...}, 128-byte swizzle, zero fill out of bounds.
static int encode(CUtensorMap* m, const void* base, int rank, const cuuint64_t* dims,
                  const cuuint64_t* strides, const cuuint32_t* box) {
  EncodeTiledFnTc enc = encode_fn();
  if (enc == nullptr) return -1;
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(base), dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : 100 + (int)r;
}

int launch_prefill_attention_tc(const PrefillAttnArgs& a, int B, cudaStream_t s, bool pair_heads) {
  if (a.key_lo != nullptr || a.key_hi != nullptr) return 1;  // padding masks: mma.sync kernel
  if (a.D != kTcD || a.q_len <= 0 || B <= 0 || a.nq % a.nkv != 0) return 1;
  TcMaps mp;
  {  // q [B, q_len, nq, D]
    cuuint64_t dims[4] = {(cuuint64_t)kTcD, (cuuint64_t)a.nq, (cuuint64_t)a.q_len, (cuuint64_t)B};
    cuuint64_t str[3] = {(cuuint64_t)kTcD * 2, (cuuint64_t)a.nq * kTcD * 2,
                         (cuuint64_t)a.q_len * a.nq * kTcD * 2};
    cuuint32_t box[4] = {64, 1, (cuuint32_t)kTcBM, 1};
    int e = encode(&mp.q, a.q, 4, dims, str, box);
    if (e) return e;
  }
  const cuuint64_t planes = (cuuint64_t)(a.batch_offset + B) * a.nkv;
  cuuint64_t kdims[3] = {(cuuint64_t)kTcD, (cuuint64_t)a.s_max, planes};
  cuuint64_t kstr[2] = {(cuuint64_t)kTcD * 2, (cuuint64_t)a.s_max * kTcD * 2};
  cuuint32_t kbox[3] = {64, (cuuint32_t)kTcBN, 1};
  int e = encode(&mp.k, a.k_cache, 3, kdims, kstr, kbox);
  if (e) return e;
  e = encode(&mp.v, a.v_cache, 3, kdims, kstr, kbox);
  if (e) return e;
  const int n_qt = (a.q_len + kTcBM - 1) / kTcBM;
  if (pair_heads && (a.nq / a.nkv) % 2 == 0) {
    // two heads of one kv group per CTA; 1-D grid, heaviest query tiles first
    const cudaError_t r =
        set_max_dynamic_smem(reinterpret_cast<const void*>(prefill_attention_tc2_kernel), kP2Smem);
    if (r != cudaSuccess) return (int)r;
    const long long blocks = (long long)n_qt * (a.nq / 2) * B;
    if (blocks > 0x7fffffff) return 1;
    return (int)launch_k(prefill_attention_tc2_kernel, dim3((unsigned)blocks), dim3(kP2Threads),
                         kP2Smem, s, mp.q, mp.k, mp.v, a);
  }
  const cudaError_t r =
      set_max_dynamic_smem(reinterpret_cast<const void*>(prefill_attention_tc_kernel), kTcSmem);
  if (r != cudaSuccess) return (int)r;
  dim3 grid(n_qt, a.nq, B);
  return (int)launch_k(prefill_attention_tc_kernel, grid, dim3(kTcThreads), kTcSmem, s, mp.q,
                       mp.k, mp.v, a);
}

}  // namespace afd
