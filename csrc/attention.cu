// GQA attention over the preallocated KV cache [B_max, n_kv, S_max, D].
//
// decode_attention_kernel: one query token per sequence. One CTA per
//   (sequence, kv head, kv split) serves the G = nq / nkv query heads that
//   share the kv head, streaming 64-key tiles of K and V through shared
//   memory with an online softmax. With more than one split, partial
//   (unnormalised O, running max, running sum) go to a workspace and
//   decode_combine_kernel merges them.
//
// prefill_attention_kernel: causal flash attention (online softmax) for
//   q_len queries per sequence that sit at positions start_pos .. start_pos +
//   q_len - 1 and see keys 0 .. their own position. bf16 m16n8k16 tensor-core
//   MMA from registers, 64 queries x 64 keys per step, 4 warps x 16 rows.
//
// start_pos is read from device memory so a captured CUDA graph replays
// correctly as the cache grows.

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "kernels.h"

namespace afd {

// =============================================================== decode ===
constexpr int kDecKeys = 64;

template <int G, int D>
__global__ void __launch_bounds__(D) decode_attention_kernel(DecodeAttnArgs a) {
  pdl_wait();
  pdl_trigger();
  constexpr int NT = D;          // threads
  constexpr int NW = NT / 32;
  constexpr int KP = D + 8;      // padded K row (conflict-free row-per-thread reads)
  __shared__ float q_s[G][D];
  __shared__ __align__(16) __nv_bfloat16 k_s[kDecKeys][KP];
  __shared__ __align__(16) __nv_bfloat16 v_s[kDecKeys][D];
  __shared__ float p_s[G][kDecKeys];
  __shared__ float alpha_s[G];
  __shared__ float m_s[G], l_s[G];

  const int b = blockIdx.x;
  const int kvh = blockIdx.y;
  const int split = blockIdx.z;
  const int nsplit = gridDim.z;
  const int tid = threadIdx.x;
  const int warp = tid / 32, lane = tid % 32;
  int kv_len = *a.start_pos + 1;
  if (kv_len < 1 || kv_len > a.s_max) {
    // the position lies outside the cache rows: read nothing, output zeros
    if (tid == 0 && b == 0 && kvh == 0 && split == 0)
      report_status(a.status, kBoundsViolation, 60);
    kv_len = 0;
  }
  const int cb = a.batch_offset + b;
  const float scale = rsqrtf((float)D);

  // key range of this split (whole tiles)
  const int n_tiles = (kv_len + kDecKeys - 1) / kDecKeys;
  const int tiles_per = (n_tiles + nsplit - 1) / nsplit;
  const int t0 = split * tiles_per;
  const int t1 = min(n_tiles, t0 + tiles_per);

  for (int i = tid; i < G * D; i += NT) {
    const int h = i / D, d = i % D;
    q_s[h][d] = bf16_to_f(a.q[((size_t)b * a.nq + kvh * G + h) * D + d]) * scale;
  }
  if (tid < G) { m_s[tid] = -INFINITY; l_s[tid] = 0.f; }
  float o[G];
#pragma unroll
  for (int h = 0; h < G; ++h) o[h] = 0.f;

  const __nv_bfloat16* kbase = a.k_cache + ((size_t)cb * a.nkv + kvh) * a.s_max * D;
  const __nv_bfloat16* vbase = a.v_cache + ((size_t)cb * a.nkv + kvh) * a.s_max * D;
  __syncthreads();

  for (int tile = t0; tile < t1; ++tile) {
    const int key0 = tile * kDecKeys;
    const int nk = min(kDecKeys, kv_len - key0);
    // load K, V tile (16-byte vectors)
    constexpr int VPR = D / 8;  // vectors per row
    for (int i = tid; i < kDecKeys * VPR; i += NT) {
      const int r = i / VPR, c = (i % VPR) * 8;
      uint4 kv = make_uint4(0, 0, 0, 0), vv = make_uint4(0, 0, 0, 0);
      if (r < nk) {
        kv = *reinterpret_cast<const uint4*>(kbase + (size_t)(key0 + r) * D + c);
        vv = *reinterpret_cast<const uint4*>(vbase + (size_t)(key0 + r) * D + c);
      }
      *reinterpret_cast<uint4*>(&k_s[r][c]) = kv;
      *reinterpret_cast<uint4*>(&v_s[r][c]) = vv;
    }
    __syncthreads();
    // scores
    for (int i = tid; i < G * kDecKeys; i += NT) {
      const int h = i / kDecKeys, k = i % kDecKeys;
      float s = -INFINITY;
      if (k < nk) {
        s = 0.f;
#pragma unroll 8
        for (int d = 0; d < D; d += 2) {
          const float2 kk = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&k_s[k][d]));
          s += q_s[h][d] * kk.x + q_s[h][d + 1] * kk.y;
        }
      }
      p_s[h][k] = s;
    }
    __syncthreads();
    // online softmax, one warp per head
    for (int h = warp; h < G; h += NW) {
      float mx = -INFINITY;
      for (int k = lane; k < kDecKeys; k += 32) mx = fmaxf(mx, p_s[h][k]);
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffff, mx, 16));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffff, mx, 8));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffff, mx, 4));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffff, mx, 2));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffff, mx, 1));
      const float m_old = m_s[h];
      const float m_new = fmaxf(m_old, mx);
      float sum = 0.f;
      for (int k = lane; k < kDecKeys; k += 32) {
        const float p = (p_s[h][k] == -INFINITY) ? 0.f : __expf(p_s[h][k] - m_new);
        p_s[h][k] = p;
        sum += p;
      }
      sum += __shfl_xor_sync(0xffffffff, sum, 16);
      sum += __shfl_xor_sync(0xffffffff, sum, 8);
      sum += __shfl_xor_sync(0xffffffff, sum, 4);
      sum += __shfl_xor_sync(0xffffffff, sum, 2);
      sum += __shfl_xor_sync(0xffffffff, sum, 1);
      if (lane == 0) {
        const float al = (m_old == -INFINITY) ? 0.f : __expf(m_old - m_new);
        alpha_s[h] = al;
        l_s[h] = l_s[h] * al + sum;
        m_s[h] = m_new;
      }
    }
    __syncthreads();
    // O += P V, thread = output dim
#pragma unroll
    for (int h = 0; h < G; ++h) o[h] *= alpha_s[h];
    for (int k = 0; k < nk; ++k) {
      const float v = bf16_to_f(v_s[k][tid]);
#pragma unroll
      for (int h = 0; h < G; ++h) o[h] += p_s[h][k] * v;
    }
    __syncthreads();
  }

  if (nsplit == 1) {
#pragma unroll
    for (int h = 0; h < G; ++h) {
      const float l = l_s[h];
      a.out[((size_t)b * a.nq + kvh * G + h) * D + tid] = f_to_bf16(l > 0.f ? o[h] / l : 0.f);
    }
  } else {
    // workspace: o_part [B, nq, nsplit, D], ml_part [B, nq, nsplit, 2]
#pragma unroll
    for (int h = 0; h < G; ++h) {
      const size_t hq = (size_t)b * a.nq + kvh * G + h;
      a.o_part[(hq * nsplit + split) * D + tid] = o[h];
      if (tid == 0) {
        a.ml_part[(hq * nsplit + split) * 2 + 0] = m_s[h];
        a.ml_part[(hq * nsplit + split) * 2 + 1] = l_s[h];
      }
    }
  }
}

// Merge split partials: one CTA of D threads per (sequence, q head).
__global__ void decode_combine_kernel(DecodeAttnArgs a, int nsplit, int D) {
  pdl_wait();
  pdl_trigger();
  const size_t hq = blockIdx.x;
  const int d = threadIdx.x;
  float m = -INFINITY;
  for (int s = 0; s < nsplit; ++s) m = fmaxf(m, a.ml_part[(hq * nsplit + s) * 2]);
  float l = 0.f, o = 0.f;
  for (int s = 0; s < nsplit; ++s) {
    const float ms = a.ml_part[(hq * nsplit + s) * 2];
    if (ms == -INFINITY) continue;
    const float w = __expf(ms - m);
    l += a.ml_part[(hq * nsplit + s) * 2 + 1] * w;
    o += a.o_part[(hq * nsplit + s) * D + d] * w;
  }
  a.out[hq * D + d] = f_to_bf16(l > 0.f ? o / l : 0.f);
}

// ============================================================== prefill ===
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma_bf16_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                               uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

constexpr int kPBM = 64;   // queries per CTA
constexpr int kPBN = 64;   // keys per step

template <int D>
__global__ void __launch_bounds__(128) prefill_attention_kernel(PrefillAttnArgs a) {
  pdl_wait();
  pdl_trigger();
  constexpr int P = D + 8;  // padded smem row (ldmatrix conflict-free)
  extern __shared__ __align__(16) uint8_t psm[];
  __nv_bfloat16* q_s = reinterpret_cast<__nv_bfloat16*>(psm);
  __nv_bfloat16* k_s = q_s + kPBM * P;
  __nv_bfloat16* v_s = k_s + kPBN * P;

  const int qtile = blockIdx.x;
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int G = a.nq / a.nkv;
  const int kvh = h / G;
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int start = *a.start_pos;
  const int q0 = qtile * kPBM;
  if (q0 >= a.q_len) return;
  const int nq_rows = min(kPBM, a.q_len - q0);
  const int cb = a.batch_offset + b;
  constexpr int VPR = D / 8;

  // Q tile -> smem
  for (int i = tid; i < kPBM * VPR; i += 128) {
    const int r = i / VPR, c = (i % VPR) * 8;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < nq_rows)
      v = *reinterpret_cast<const uint4*>(
          a.q + (((size_t)b * a.q_len + q0 + r) * a.nq + h) * D + c);
    *reinterpret_cast<uint4*>(q_s + r * P + c) = v;
  }
  __syncthreads();
  // Q fragments for this warp's 16 rows
  uint32_t qf[D / 16][4];
  {
    const int r = warp * 16 + (lane % 16);
    const int cofs = (lane / 16) * 8;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      const uint32_t addr = smem_u32(q_s + r * P + kk * 16 + cofs);
      ldsm_x4(addr, qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
    }
  }
  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const float sl2 = rsqrtf((float)D) * 1.4426950408889634f;
  // query positions of this thread's two rows
  const int qr0 = warp * 16 + lane / 4;
  const int qpos0 = start + q0 + qr0;
  const int qpos1 = qpos0 + 8;
  const int kv_end = start + q0 + nq_rows;  // exclusive
  // visible key range (padding): [key_lo, key_hi) of this cache row
  const int key_lo = a.key_lo != nullptr ? a.key_lo[cb] : 0;
  const int key_hi = a.key_hi != nullptr ? a.key_hi[cb] : kv_end;
  const __nv_bfloat16* kbase = a.k_cache + ((size_t)cb * a.nkv + kvh) * a.s_max * D;
  const __nv_bfloat16* vbase = a.v_cache + ((size_t)cb * a.nkv + kvh) * a.s_max * D;

  for (int k0 = 0; k0 < kv_end; k0 += kPBN) {
    const int nk = min(kPBN, kv_end - k0);
    __syncthreads();
    for (int i = tid; i < kPBN * VPR; i += 128) {
      const int r = i / VPR, c = (i % VPR) * 8;
      uint4 kv = make_uint4(0, 0, 0, 0), vv = make_uint4(0, 0, 0, 0);
      if (r < nk) {
        kv = *reinterpret_cast<const uint4*>(kbase + (size_t)(k0 + r) * D + c);
        vv = *reinterpret_cast<const uint4*>(vbase + (size_t)(k0 + r) * D + c);
      }
      *reinterpret_cast<uint4*>(k_s + r * P + c) = kv;
      *reinterpret_cast<uint4*>(v_s + r * P + c) = vv;
    }
    __syncthreads();
    // S = Q K^T : 16 x 64 per warp -> 8 n-tiles
    float s[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {  // pairs of n-tiles (16 keys)
        // matrices: keys np*16+[0,8) d[kk*16, +8), same keys d+8, keys+8 d, keys+8 d+8
        const int key = np * 16 + (lane % 8) + ((lane / 16) * 8);
        const int dofs = kk * 16 + ((lane / 8) % 2) * 8;
        uint32_t r0, r1, r2, r3;
        ldsm_x4(smem_u32(k_s + key * P + dofs), r0, r1, r2, r3);
        mma_bf16_16816(s[np * 2], qf[kk], r0, r1);
        mma_bf16_16816(s[np * 2 + 1], qf[kk], r2, r3);
      }
    }
    // mask + online softmax (rows qr0 and qr0 + 8)
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const int kc = k0 + nt * 8 + (lane % 4) * 2;
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int kp = kc + e;
        float v0 = s[nt][e] * sl2, v1 = s[nt][2 + e] * sl2;
        const bool hidden = kp >= kv_end || kp < key_lo || kp >= key_hi;
        if (kp > qpos0 || hidden) v0 = -INFINITY;
        if (kp > qpos1 || hidden) v1 = -INFINITY;
        s[nt][e] = v0;
        s[nt][2 + e] = v1;
        mx0 = fmaxf(mx0, v0);
        mx1 = fmaxf(mx1, v1);
      }
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffff, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffff, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffff, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffff, mx1, 2));
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float al0 = (mn0 == -INFINITY) ? 1.f : exp2f(m0 - mn0);
    const float al1 = (mn1 == -INFINITY) ? 1.f : exp2f(m1 - mn1);
    float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float p0 = (s[nt][e] == -INFINITY) ? 0.f : exp2f(s[nt][e] - mn0);
        const float p1 = (s[nt][2 + e] == -INFINITY) ? 0.f : exp2f(s[nt][2 + e] - mn1);
        s[nt][e] = p0;
        s[nt][2 + e] = p1;
        rs0 += p0;
        rs1 += p1;
      }
    }
    rs0 += __shfl_xor_sync(0xffffffff, rs0, 1);
    rs0 += __shfl_xor_sync(0xffffffff, rs0, 2);
    rs1 += __shfl_xor_sync(0xffffffff, rs1, 1);
    rs1 += __shfl_xor_sync(0xffffffff, rs1, 2);
    l0 = l0 * al0 + rs0;
    l1 = l1 * al1 + rs1;
    m0 = mn0;
    m1 = mn1;
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      o[i][0] *= al0; o[i][1] *= al0;
      o[i][2] *= al1; o[i][3] *= al1;
    }
    // O += P V : k = keys (4 steps of 16), n = D (D/8 tiles)
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t pa[4];
      pa[0] = pack_bf16x2(s[kk * 2][0], s[kk * 2][1]);
      pa[1] = pack_bf16x2(s[kk * 2][2], s[kk * 2][3]);
      pa[2] = pack_bf16x2(s[kk * 2 + 1][0], s[kk * 2 + 1][1]);
      pa[3] = pack_bf16x2(s[kk * 2 + 1][2], s[kk * 2 + 1][3]);
#pragma unroll
      for (int dp = 0; dp < D / 16; ++dp) {
        // transposed loads: keys kk*16+[0,16), dims dp*16+[0,16)
        const int key = kk * 16 + (lane % 8) + ((lane / 8) % 2) * 8;
        const int dofs = dp * 16 + (lane / 16) * 8;
        uint32_t r0, r1, r2, r3;
        ldsm_x4_t(smem_u32(v_s + key * P + dofs), r0, r1, r2, r3);
        mma_bf16_16816(o[dp * 2], pa, r0, r1);
        mma_bf16_16816(o[dp * 2 + 1], pa, r2, r3);
      }
    }
  }
  // write O (rows qr0, qr0 + 8)
  const float inv0 = l0 > 0.f ? 1.f / l0 : 0.f;
  const float inv1 = l1 > 0.f ? 1.f / l1 : 0.f;
#pragma unroll
  for (int nt = 0; nt < D / 8; ++nt) {
    const int d = nt * 8 + (lane % 4) * 2;
    if (qr0 < nq_rows) {
      __nv_bfloat16* dst = a.out + (((size_t)b * a.q_len + q0 + qr0) * a.nq + h) * D + d;
      *reinterpret_cast<uint32_t*>(dst) = pack_bf16x2(o[nt][0] * inv0, o[nt][1] * inv0);
    }
    if (qr0 + 8 < nq_rows) {
      __nv_bfloat16* dst = a.out + (((size_t)b * a.q_len + q0 + qr0 + 8) * a.nq + h) * D + d;
      *reinterpret_cast<uint32_t*>(dst) = pack_bf16x2(o[nt][2] * inv1, o[nt][3] * inv1);
    }
  }
}

// ================================================= fused decode attention ===
// One CTA per (sequence, kv head), 8 warps. Prologue (optional): the CTA
// itself applies q/k RMSNorm + RoPE to its G query heads and its kv head for
// the new token and appends k, v to the cache (the qk_norm_rope_cache kernel
// folded in). Main loop: warp w takes 32-key tiles w, w+8, ... of the cache:
// cp.async into a warp-private padded tile, S = Q K^T and O += P V on m16n8k16
// tensor-core MMAs with the G query heads as rows (padded to 16), online
// softmax in the log2 domain. Epilogue: the 8 warps' (m, l, O) merge in
// shared memory -- no split workspace and no second kernel.
constexpr int kFdWarps = 8;
constexpr int kFdKeys = 32;

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gsrc)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
}

// q/k head: RMSNorm over D, then RoPE at `pos`; lane owns pairs (j, j+D/2),
// j = lane + 32 i. Rounds like HF (bf16 after norm, weight, each product).
template <int D>
__device__ __forceinline__ void norm_rope_head(const __nv_bfloat16* src, const __nv_bfloat16* nw,
                                               const float* rope, int pos, float eps, int lane,
                                               float (&lo)[D / 64], float (&hi)[D / 64]) {
  constexpr int half = D / 2;
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < D / 64; ++i) {
    lo[i] = bf16_to_f(src[lane + 32 * i]);
    hi[i] = bf16_to_f(src[half + lane + 32 * i]);
    ss += lo[i] * lo[i] + hi[i] * hi[i];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffff, ss, o);
  const float rstd = rsqrtf(ss / (float)D + eps);
#pragma unroll
  for (int i = 0; i < D / 64; ++i) {
    const int j = lane + 32 * i;
    const float xl = round_bf16(bf16_to_f(nw[j]) * round_bf16(lo[i] * rstd));
    const float xh = round_bf16(bf16_to_f(nw[half + j]) * round_bf16(hi[i] * rstd));
    const float c = rope[(size_t)pos * D + j];
    const float s = rope[(size_t)pos * D + half + j];
    lo[i] = round_bf16(round_bf16(xl * c) + round_bf16(-xh * s));
    hi[i] = round_bf16(round_bf16(xh * c) + round_bf16(xl * s));
  }
}

template <int G, int D>
__global__ void __launch_bounds__(kFdWarps * 32) decode_attention_fused_kernel(FusedDecodeArgs a) {
  pdl_wait();
  pdl_trigger();
  constexpr int P = D + 8;                 // padded row (ldmatrix conflict-free)
  constexpr int TILE = kFdKeys * P;        // elements per K or V tile
  extern __shared__ __align__(16) uint8_t fsm[];
  __nv_bfloat16* q_s = reinterpret_cast<__nv_bfloat16*>(fsm);          // [16][P]
  __nv_bfloat16* kv_s = q_s + 16 * P;                                  // [warps][2][32][P]
  const int b = blockIdx.x;
  const int kvh = blockIdx.y;
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int pos = *a.start_pos;
  const int kv_len = pos + 1;
  const int cb = a.batch_offset + b;
  if (pos < 0 || pos >= a.s_max) {
    // no cache row for the new token: write nothing to the cache, output zeros
    if (tid == 0 && b == 0 && kvh == 0) report_status(a.status, kBoundsViolation, 61);
    for (int i = tid; i < G * D; i += blockDim.x)
      a.out[((size_t)b * a.nq + kvh * G) * D + i] = f_to_bf16(0.f);
    return;
  }
  __nv_bfloat16* kbase = a.k_cache + ((size_t)cb * a.nkv + kvh) * a.s_max * D;
  __nv_bfloat16* vbase = a.v_cache + ((size_t)cb * a.nkv + kvh) * a.s_max * D;

  // ---------------------------------------------------------------- Q (+K/V)
  for (int i = tid; i < 16 * P; i += blockDim.x) q_s[i] = f_to_bf16(0.f);
  __syncthreads();
  if (a.qkv != nullptr) {
    const __nv_bfloat16* row = a.qkv + (size_t)b * a.ld_qkv;
    for (int hr = warp; hr < G + 2; hr += kFdWarps) {
      float lo[D / 64], hi[D / 64];
      if (hr < G + 1) {
        const bool is_q = hr < G;
        const int head = is_q ? kvh * G + hr : a.nq + kvh;
        norm_rope_head<D>(row + (size_t)head * D, is_q ? a.q_norm : a.k_norm, a.rope, pos,
                          a.eps, lane, lo, hi);
        __nv_bfloat16* dst = is_q ? q_s + hr * P : kbase + (size_t)pos * D;
#pragma unroll
        for (int i = 0; i < D / 64; ++i) {
          dst[lane + 32 * i] = f_to_bf16(lo[i]);
          dst[D / 2 + lane + 32 * i] = f_to_bf16(hi[i]);
        }
      } else {  // value head: copy into the cache
        const __nv_bfloat16* src = row + (size_t)(a.nq + a.nkv + kvh) * D;
        for (int j = lane; j < D; j += 32) vbase[(size_t)pos * D + j] = src[j];
      }
    }
    __threadfence_block();
  } else {
    for (int i = tid; i < G * D; i += blockDim.x)
      q_s[(i / D) * P + i % D] = a.q[((size_t)b * a.nq + kvh * G) * D + i];
  }
  __syncthreads();

  uint32_t qf[D / 16][4];
  {
    const int r = lane % 16, cofs = (lane / 16) * 8;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk)
      ldsm_x4(smem_u32(q_s + r * P + kk * 16 + cofs), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
  }
  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const float sl2 = rsqrtf((float)D) * 1.4426950408889634f;
  __nv_bfloat16* ks = kv_s + warp * 2 * TILE;
  __nv_bfloat16* vs = ks + TILE;
  const int n_tiles = (kv_len + kFdKeys - 1) / kFdKeys;
  constexpr int VPR = D / 8;

  for (int tile = warp; tile < n_tiles; tile += kFdWarps) {
    const int key0 = tile * kFdKeys;
    const int nk = min(kFdKeys, kv_len - key0);
    for (int i = lane; i < kFdKeys * VPR; i += 32) {
      const int r = i / VPR, c = (i % VPR) * 8;
      if (r < nk) {
        cp_async16(ks + r * P + c, kbase + (size_t)(key0 + r) * D + c);
        cp_async16(vs + r * P + c, vbase + (size_t)(key0 + r) * D + c);
      } else {
        *reinterpret_cast<uint4*>(ks + r * P + c) = make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(vs + r * P + c) = make_uint4(0, 0, 0, 0);
      }
    }
    cp_async_wait_all();
    __syncwarp();
    float s[4][4];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
#pragma unroll
      for (int np = 0; np < 2; ++np) {
        const int key = np * 16 + (lane % 8) + ((lane / 16) * 8);
        const int dofs = kk * 16 + ((lane / 8) % 2) * 8;
        uint32_t r0, r1, r2, r3;
        ldsm_x4(smem_u32(ks + key * P + dofs), r0, r1, r2, r3);
        mma_bf16_16816(s[np * 2], qf[kk], r0, r1);
        mma_bf16_16816(s[np * 2 + 1], qf[kk], r2, r3);
      }
    }
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const bool valid = nt * 8 + (lane % 4) * 2 + e < nk;
        const float v0 = valid ? s[nt][e] * sl2 : -INFINITY;
        const float v1 = valid ? s[nt][2 + e] * sl2 : -INFINITY;
        s[nt][e] = v0;
        s[nt][2 + e] = v1;
        mx0 = fmaxf(mx0, v0);
        mx1 = fmaxf(mx1, v1);
      }
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffff, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffff, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffff, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffff, mx1, 2));
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float al0 = (mn0 == -INFINITY) ? 1.f : exp2f(m0 - mn0);
    const float al1 = (mn1 == -INFINITY) ? 1.f : exp2f(m1 - mn1);
    float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float p0 = (s[nt][e] == -INFINITY) ? 0.f : exp2f(s[nt][e] - mn0);
        const float p1 = (s[nt][2 + e] == -INFINITY) ? 0.f : exp2f(s[nt][2 + e] - mn1);
        s[nt][e] = p0;
        s[nt][2 + e] = p1;
        rs0 += p0;
        rs1 += p1;
      }
    }
    rs0 += __shfl_xor_sync(0xffffffff, rs0, 1);
    rs0 += __shfl_xor_sync(0xffffffff, rs0, 2);
    rs1 += __shfl_xor_sync(0xffffffff, rs1, 1);
    rs1 += __shfl_xor_sync(0xffffffff, rs1, 2);
    l0 = l0 * al0 + rs0;
    l1 = l1 * al1 + rs1;
    m0 = mn0;
    m1 = mn1;
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      o[i][0] *= al0; o[i][1] *= al0;
      o[i][2] *= al1; o[i][3] *= al1;
    }
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) {
      uint32_t pa[4];
      pa[0] = pack_bf16x2(s[kk * 2][0], s[kk * 2][1]);
      pa[1] = pack_bf16x2(s[kk * 2][2], s[kk * 2][3]);
      pa[2] = pack_bf16x2(s[kk * 2 + 1][0], s[kk * 2 + 1][1]);
      pa[3] = pack_bf16x2(s[kk * 2 + 1][2], s[kk * 2 + 1][3]);
#pragma unroll
      for (int dp = 0; dp < D / 16; ++dp) {
        const int key = kk * 16 + (lane % 8) + ((lane / 8) % 2) * 8;
        const int dofs = dp * 16 + (lane / 16) * 8;
        uint32_t r0, r1, r2, r3;
        ldsm_x4_t(smem_u32(vs + key * P + dofs), r0, r1, r2, r3);
        mma_bf16_16816(o[dp * 2], pa, r0, r1);
        mma_bf16_16816(o[dp * 2 + 1], pa, r2, r3);
      }
    }
    __syncwarp();
  }

  // ------------------------------------------------------ merge 8 warps
  __syncthreads();  // tiles no longer needed: reuse their smem
  float* wm = reinterpret_cast<float*>(kv_s);          // [warps][16]
  float* wl = wm + kFdWarps * 16;                      // [warps][16]
  float* wo = wl + kFdWarps * 16;                      // [warps][G][D]
  const int r0 = lane / 4, r1 = r0 + 8;
  if (lane % 4 == 0) {
    wm[warp * 16 + r0] = m0; wl[warp * 16 + r0] = l0;
    wm[warp * 16 + r1] = m1; wl[warp * 16 + r1] = l1;
  }
#pragma unroll
  for (int nt = 0; nt < D / 8; ++nt) {
    const int d = nt * 8 + (lane % 4) * 2;
    if (r0 < G) {
      wo[(warp * G + r0) * D + d] = o[nt][0];
      wo[(warp * G + r0) * D + d + 1] = o[nt][1];
    }
    if (r1 < G) {
      wo[(warp * G + r1) * D + d] = o[nt][2];
      wo[(warp * G + r1) * D + d + 1] = o[nt][3];
    }
  }
  __syncthreads();
  for (int i = tid; i < G * D; i += blockDim.x) {
    const int h = i / D, d = i % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kFdWarps; ++w) M = fmaxf(M, wm[w * 16 + h]);
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < kFdWarps; ++w) {
      const float mw = wm[w * 16 + h];
      if (mw == -INFINITY) continue;
      const float sc = exp2f(mw - M);
      L += wl[w * 16 + h] * sc;
      O += wo[(w * G + h) * D + d] * sc;
    }
    a.out[((size_t)b * a.nq + kvh * G + h) * D + d] = f_to_bf16(L > 0.f ? O / L : 0.f);
  }
}

template <int G, int D>
static int fused_launch(const FusedDecodeArgs& a, int B, cudaStream_t s) {
  constexpr int P = D + 8;
  const int smem = (16 * P + kFdWarps * 2 * kFdKeys * P) * 2;
  static_assert((kFdWarps * 2 * kFdKeys * (D + 8)) * 2 >=
                    (2 * kFdWarps * 16 + kFdWarps * G * D) * 4,
                "merge buffers must fit in the tile region");
  const cudaError_t e = set_max_dynamic_smem(
      reinterpret_cast<const void*>(decode_attention_fused_kernel<G, D>), smem);
  if (e != cudaSuccess) return (int)e;
  return (int)launch_k(decode_attention_fused_kernel<G, D>, dim3(B, a.nkv), dim3(kFdWarps * 32), smem, s, a);
}

int launch_decode_attention_fused(const FusedDecodeArgs& a, int B, cudaStream_t s) {
  if (B == 0) return 0;
  const int G = a.nq / a.nkv;
  if (G == 8 && a.D == 128) return fused_launch<8, 128>(a, B, s);
  if (G == 2 && a.D == 64) return fused_launch<2, 64>(a, B, s);
  if (G == 4 && a.D == 128) return fused_launch<4, 128>(a, B, s);
  if (G == 8 && a.D == 64) return fused_launch<8, 64>(a, B, s);
  return 1;
}

// ============================================================= launchers ===
template <int G, int D>
static void dec_launch(const DecodeAttnArgs& a, int B, int nsplit, cudaStream_t s) {
  dim3 grid(B, a.nkv, nsplit);
  launch_k(decode_attention_kernel<G, D>, grid, dim3(D), 0, s, a);
}

int launch_decode_attention(const DecodeAttnArgs& a, int B, int nsplit, cudaStream_t s) {
  if (B == 0) return 0;
  const int G = a.nq / a.nkv;
  if (nsplit > 1 && (a.o_part == nullptr || a.ml_part == nullptr)) return 2;
  if (G == 8 && a.D == 128) dec_launch<8, 128>(a, B, nsplit, s);
  else if (G == 2 && a.D == 64) dec_launch<2, 64>(a, B, nsplit, s);
  else if (G == 4 && a.D == 128) dec_launch<4, 128>(a, B, nsplit, s);
  else if (G == 8 && a.D == 64) dec_launch<8, 64>(a, B, nsplit, s);
  else return 1;
  if (nsplit > 1) launch_k(decode_combine_kernel, dim3(B * a.nq), dim3(a.D), 0, s, a, nsplit, a.D);
  return (int)cudaGetLastError();
}

int launch_prefill_attention(const PrefillAttnArgs& a, int B, cudaStream_t s) {
  if (B == 0 || a.q_len == 0) return 0;
  dim3 grid((a.q_len + kPBM - 1) / kPBM, a.nq, B);
  if (a.D == 128) {
    const int smem = (kPBM + 2 * kPBN) * (128 + 8) * 2;
    const cudaError_t e = set_max_dynamic_smem(
        reinterpret_cast<const void*>(prefill_attention_kernel<128>), smem);
    if (e != cudaSuccess) return (int)e;
    launch_k(prefill_attention_kernel<128>, grid, dim3(128), smem, s, a);
  } else if (a.D == 64) {
    const int smem = (kPBM + 2 * kPBN) * (64 + 8) * 2;
    launch_k(prefill_attention_kernel<64>, grid, dim3(128), smem, s, a);
  } else {
    return 1;
  }
  return (int)cudaGetLastError();
}

}  // namespace afd
