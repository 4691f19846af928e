// Memory-bound kernels of the Qwen3-MoE step: RMSNorm over a sum of partial
// hidden states, fused q/k RMSNorm + RoPE + KV-cache append, router
// softmax/top-k, MoE routing (histogram, prefix sums, row blocks for the
// grouped GEMM), token gather, weighted combine (+ residual, + peer stores),
// argmax, and the flag signal / bounded wait kernels.
//
// Numerics follow HF Qwen3-MoE: fp32 math with a bf16 rounding at every point
// where the eager PyTorch code materialises a bf16 tensor.

#include <cstdlib>

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "kernels.h"

namespace afd {

// ------------------------------------------------------------ helpers ---
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffff, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffff, v, o));
  return v;
}

template <int NT>
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x / 32, l = threadIdx.x % 32;
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = (l < NT / 32) ? red[l] : 0.f;
  t = warp_sum(t);
  __syncthreads();
  return t;
}

struct Vec8 {
  uint4 u;
};

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&f)[8]) {
  uint4 u = *reinterpret_cast<const uint4*>(p);
  unpack_bf16x2(u.x, f[0], f[1]);
  unpack_bf16x2(u.y, f[2], f[3]);
  unpack_bf16x2(u.z, f[4], f[5]);
  unpack_bf16x2(u.w, f[6], f[7]);
}

__device__ __forceinline__ void store8(__nv_bfloat16* p, const float (&f)[8]) {
  uint4 u;
  u.x = pack_bf16x2(f[0], f[1]);
  u.y = pack_bf16x2(f[2], f[3]);
  u.z = pack_bf16x2(f[4], f[5]);
  u.w = pack_bf16x2(f[6], f[7]);
  *reinterpret_cast<uint4*>(p) = u;
}

// ------------------------------------------------------- sum + RMSNorm ---
// x = sum_p parts[p][row] (fp32 sum, one bf16 rounding); y = w * bf16(x * rstd)
// One CTA (256 threads) per row; H % 8 == 0, H <= 256 * 8 * 4.
constexpr int kNormThreads = 256;

// Every CTA: thread 0 waits (bounded) for the flags, then the CTA proceeds.
// The acquire load plus the barrier order the peers' data stores before this
// CTA's reads. On a timeout the status word records it and the CTA proceeds
// (the host turns the status into an error after the step).
__device__ __forceinline__ void block_wait(const FlagWait& w, int where) {
  if (w.n == 0) return;
  if (threadIdx.x == 0) {
    const int v = w.value + (w.epoch != nullptr ? *w.epoch : 0);
    for (int i = 0; i < w.n; ++i)
      if (!wait_flag_geq(w.flags[i], v, w.status, where + i, w.timeout_ns)) break;
  }
  __syncthreads();
}

__global__ void __launch_bounds__(kNormThreads) sum_rmsnorm_kernel(SumNormArgs a) {
  __shared__ float red[kNormThreads / 32];
  pdl_wait();
  pdl_trigger();
  block_wait(a.wait, 120);
  const int row = blockIdx.x;
  const int H = a.H;
  constexpr int kMaxChunks = 4;
  float xv[kMaxChunks][8];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < kMaxChunks; ++c) {
    const int col = (c * kNormThreads + threadIdx.x) * 8;
    if (col < H) {
      // every part's vector is requested before the sum (loads in flight)
      uint4 pv[kMaxParts];
#pragma unroll
      for (int p = 0; p < kMaxParts; ++p)
        pv[p] = p < a.n_parts
                    ? *reinterpret_cast<const uint4*>(a.parts[p] + (size_t)row * a.ld_in + col)
                    : make_uint4(0, 0, 0, 0);
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int p = 0; p < kMaxParts; ++p) {
        if (p >= a.n_parts) break;
        const uint32_t* q = &pv[p].x;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float u0, u1;
          unpack_bf16x2(q[e], u0, u1);
          acc[2 * e] += u0;
          acc[2 * e + 1] += u1;
        }
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        xv[c][i] = round_bf16(acc[i]);
        ss += xv[c][i] * xv[c][i];
      }
      if (a.x_out != nullptr) store8(a.x_out + (size_t)row * H + col, xv[c]);
    }
  }
  const float tot = block_sum<kNormThreads>(ss, red);
  const float rstd = rsqrtf(tot / (float)H + a.eps);
#pragma unroll
  for (int c = 0; c < kMaxChunks; ++c) {
    const int col = (c * kNormThreads + threadIdx.x) * 8;
    if (col < H) {
      float w[8], y[8];
      load8(a.weight + col, w);
#pragma unroll
      for (int i = 0; i < 8; ++i) y[i] = w[i] * round_bf16(xv[c][i] * rstd);
      store8(a.y_out + (size_t)row * a.ld_out + col, y);
    }
  }
}

// --------------------------------------- q/k RMSNorm + RoPE + KV append ---
// One warp per (token, head); heads [0, nq) are queries, [nq, nq+nkv) keys,
// [nq+nkv, nq+2nkv) values (copied to the cache unchanged). Lane l owns the
// rotation pairs (j, j + D/2) for j = l + 32 * i.
__global__ void qk_norm_rope_cache_kernel(QKRopeArgs a) {
  pdl_wait();
  pdl_trigger();
  const int warps_per_block = blockDim.x / 32;
  const int gw = blockIdx.x * warps_per_block + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int n_heads = a.nq + 2 * a.nkv;
  if (gw >= a.T * n_heads) return;
  const int t = gw / n_heads;
  const int h = gw % n_heads;
  const int D = a.D;
  const int half = D / 2;
  const int npair = half / 32;  // 1 (D=64) or 2 (D=128)
  const int start = *a.start_pos;
  const int pos = start + t % a.q_len;
  const int b = a.batch_offset + t / a.q_len;
  const __nv_bfloat16* src = a.qkv + (size_t)t * a.ld_qkv + (size_t)h * D;

  float lo[2], hi[2];
  for (int i = 0; i < npair; ++i) {
    lo[i] = bf16_to_f(src[lane + 32 * i]);
    hi[i] = bf16_to_f(src[half + lane + 32 * i]);
  }
  if (h >= a.nq + a.nkv) {  // value head: straight copy into the cache
    const int kvh = h - a.nq - a.nkv;
    __nv_bfloat16* dst = a.v_cache + (((size_t)b * a.nkv + kvh) * a.s_max + pos) * D;
    for (int i = 0; i < npair; ++i) {
      dst[lane + 32 * i] = f_to_bf16(lo[i]);
      dst[half + lane + 32 * i] = f_to_bf16(hi[i]);
    }
    return;
  }
  const bool is_q = h < a.nq;
  const __nv_bfloat16* nw = is_q ? a.q_norm : a.k_norm;
  float ss = 0.f;
  for (int i = 0; i < npair; ++i) ss += lo[i] * lo[i] + hi[i] * hi[i];
  ss = warp_sum(ss);
  const float rstd = rsqrtf(ss / (float)D + a.eps);
  for (int i = 0; i < npair; ++i) {
    const int j = lane + 32 * i;
    const float xl = round_bf16(bf16_to_f(nw[j]) * round_bf16(lo[i] * rstd));
    const float xh = round_bf16(bf16_to_f(nw[half + j]) * round_bf16(hi[i] * rstd));
    const float c = a.rope[(size_t)pos * D + j];
    const float s = a.rope[(size_t)pos * D + half + j];
    // HF: x * cos + rotate_half(x) * sin, each product and the sum in bf16
    lo[i] = round_bf16(round_bf16(xl * c) + round_bf16(-xh * s));
    hi[i] = round_bf16(round_bf16(xh * c) + round_bf16(xl * s));
  }
  __nv_bfloat16* dst;
  if (is_q) {
    dst = a.q_out + ((size_t)t * a.nq + h) * D;
  } else {
    const int kvh = h - a.nq;
    dst = a.k_cache + (((size_t)b * a.nkv + kvh) * a.s_max + pos) * D;
  }
  for (int i = 0; i < npair; ++i) {
    dst[lane + 32 * i] = f_to_bf16(lo[i]);
    dst[half + lane + 32 * i] = f_to_bf16(hi[i]);
  }
}

// ------------------------------------------------------- router top-k ---
// logits [T, E] bf16 (E <= 256) -> softmax (fp32) -> top-k -> renormalise.
// One warp per token. Ties resolve to the lower expert index.
// Softmax + top-k + renormalise of one token's router logits by one warp;
// lane 0 writes ids / weights.
__device__ __forceinline__ void topk_token(const __nv_bfloat16* logits, int E, int top_k,
                                           int renorm, int lane, int32_t* ids_out,
                                           float* w_out) {
  // Register-resident: the loops run over the compile-time bound with a guard,
  // and lane k keeps the k-th pick (top_k <= 16 < 32), so nothing is indexed
  // at run time and nothing goes to local memory.
  constexpr int kMaxPer = 8;  // E <= 256
  float v[kMaxPer];
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) {
    const int e = lane + 32 * i;
    v[i] = e < E ? bf16_to_f(logits[e]) : -INFINITY;
    m = fmaxf(m, v[i]);
  }
  m = warp_max(m);
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) {
    const int e = lane + 32 * i;
    v[i] = e < E ? __expf(v[i] - m) : 0.f;
    s += v[i];
  }
  s = warp_sum(s);
  const float inv = 1.f / s;
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) v[i] *= inv;
  float my_w = 0.f;
  int my_e = 0;
  float wsum = 0.f;  // the same on every lane: the butterfly leaves every lane the same pick
  for (int k = 0; k < top_k; ++k) {
    float best = -1.f;
    int be = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i) {
      const int e = lane + 32 * i;
      if (e < E && (v[i] > best || (v[i] == best && e < be))) { best = v[i]; be = e; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffff, best, o);
      const int oe = __shfl_xor_sync(0xffffffff, be, o);
      if (ob > best || (ob == best && oe < be)) { best = ob; be = oe; }
    }
    if (lane == k) { my_w = best; my_e = be; }
    wsum += best;
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i)
      if (lane + 32 * i == be) v[i] = -2.f;  // remove from further rounds
  }
  if (lane < top_k) {
    ids_out[lane] = my_e;
    w_out[lane] = my_w * (renorm ? 1.f / wsum : 1.f);
  }
}

// topk_token on half a warp: lanes hl = 0..15 of the half own experts
// hl + 16 i, so two tokens are ranked at once. Same picks, order, ties (the
// lower expert index first) and weights as topk_token. Both halves must call
// it together (the shuffles span the warp, 16 lanes wide); `store` = false
// ranks without writing (a half with no token).
__device__ __forceinline__ void topk_halfwarp(const __nv_bfloat16* logits, int E, int top_k,
                                              int renorm, int hl, bool store, int32_t* ids_out,
                                              float* w_out) {
  constexpr int kMaxPer = 16;  // E <= 256
  float v[kMaxPer];
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) {
    const int e = hl + 16 * i;
    v[i] = e < E ? bf16_to_f(logits[e]) : -INFINITY;
    m = fmaxf(m, v[i]);
  }
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o, 16));
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) {
    const int e = hl + 16 * i;
    v[i] = e < E ? __expf(v[i] - m) : 0.f;
    s += v[i];
  }
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o, 16);
  const float inv = 1.f / s;
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) v[i] *= inv;
  float my_w = 0.f;
  int my_e = 0;
  float wsum = 0.f;
  for (int k = 0; k < top_k; ++k) {
    float best = -1.f;
    int be = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i) {
      const int e = hl + 16 * i;
      if (e < E && (v[i] > best || (v[i] == best && e < be))) { best = v[i]; be = e; }
    }
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o, 16);
      const int oe = __shfl_xor_sync(0xffffffffu, be, o, 16);
      if (ob > best || (ob == best && oe < be)) { best = ob; be = oe; }
    }
    if (hl == k) { my_w = best; my_e = be; }
    wsum += best;
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i)
      if (hl + 16 * i == be) v[i] = -2.f;  // remove from further rounds
  }
  if (store && hl < top_k) {
    ids_out[hl] = my_e;
    w_out[hl] = my_w * (renorm ? 1.f / wsum : 1.f);
  }
}

__global__ void router_topk_kernel(RouterArgs a) {
  pdl_wait();
  pdl_trigger();
  const int warps_per_block = blockDim.x / 32;
  const int t = blockIdx.x * warps_per_block + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (t >= a.T) return;
  topk_token(a.logits + (size_t)t * a.ld_logits, a.E, a.top_k, a.renorm, lane,
             a.ids + (size_t)t * a.top_k, a.weights + (size_t)t * a.top_k);
}

// ------------------------------------------------------- MoE routing ---
// Single CTA. Counts the (token, k) pairs that land on local experts,
// assigns each a row in expert-sorted order, writes the row's source token
// and routing weight, the inverse map inv[t*k + j] (-1 if not local), the
// expert row offsets and the row-block list for the grouped GEMM
// ({row_start, n_rows, expert, 0}, at most block_n rows per block).
constexpr int kAlignThreads = 1024;
constexpr int kMaxLocalExperts = 256;

// Row and block offsets of every local expert from its row count `cnt`
// (warp-wide exclusive scans), the expert offsets, the row-block list and its
// size. Every thread of the CTA calls it after `cnt` is complete.
__device__ void scan_and_blocks(const int* cnt, int* off, int* boff, const MoeAlignArgs& a) {
  if (threadIdx.x < 32) {
    // warp-wide exclusive scans of row counts and block counts; lane l owns
    // experts [l * per, (l + 1) * per)
    const int lane = threadIdx.x;
    const int per = (a.n_local + 31) / 32;
    int rows = 0, blocks = 0;
    for (int j = 0; j < per; ++j) {
      const int e = lane * per + j;
      if (e < a.n_local) {
        rows += cnt[e];
        blocks += (cnt[e] + a.block_n - 1) / a.block_n;
      }
    }
    int rs = rows, bs = blocks;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int r2 = __shfl_up_sync(0xffffffff, rs, o);
      const int b2 = __shfl_up_sync(0xffffffff, bs, o);
      if (lane >= o) { rs += r2; bs += b2; }
    }
    int racc = rs - rows, bacc = bs - blocks;  // exclusive prefix
    for (int j = 0; j < per; ++j) {
      const int e = lane * per + j;
      if (e < a.n_local) {
        off[e] = racc;
        boff[e] = bacc;
        racc += cnt[e];
        bacc += (cnt[e] + a.block_n - 1) / a.block_n;
      }
    }
    if (lane == 31) {
      off[a.n_local] = rs;
      boff[a.n_local] = bs;
      *a.num_blocks = bs;
      *a.num_rows = rs;
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e <= a.n_local; e += blockDim.x) a.expert_offsets[e] = off[e];
  for (int e = threadIdx.x; e < a.n_local; e += blockDim.x) {
    int b = boff[e];
    for (int r = 0; r < cnt[e]; r += a.block_n, ++b)
      a.blocks[b] = make_int4(off[e] + r, min(a.block_n, cnt[e] - r), e, 0);
  }
}

// Body shared by moe_align_kernel and moe_route_kernel; every thread of the
// (single) CTA calls it. `ids` / `weights` may live in global or shared memory.
__device__ void align_body(const int32_t* ids, const float* weights, const MoeAlignArgs& a,
                           int* cnt, int* off, int* boff) {
  for (int e = threadIdx.x; e < a.n_local; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  const int n = a.T * a.top_k;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int e = ids[i] - a.expert_start;
    int slot = -1;
    if (e >= 0 && e < a.n_local) slot = atomicAdd(&cnt[e], 1);
    a.inv[i] = slot;  // provisional: slot within the expert
  }
  __syncthreads();
  scan_and_blocks(cnt, off, boff, a);
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int slot = a.inv[i];
    if (slot < 0) continue;
    const int e = ids[i] - a.expert_start;
    const int row = off[e] + slot;
    a.inv[i] = row;
    a.row_token[row] = i / a.top_k;
    a.row_weight[row] = weights[i];
  }
}

__global__ void __launch_bounds__(kAlignThreads) moe_align_kernel(MoeAlignArgs a) {
  __shared__ int cnt[kMaxLocalExperts];
  __shared__ int off[kMaxLocalExperts + 1];
  __shared__ int boff[kMaxLocalExperts + 1];
  pdl_wait();
  pdl_trigger();
  align_body(a.ids, a.weights, a, cnt, off, boff);
}

// Multi-CTA routing for large token counts (prefill): chunk c of kAlignChunk
// (token, k) entries gets its per-expert counts and provisional slots in one
// CTA (moe_align_hist_kernel); the last of those CTAs turns the counts into
// per-chunk row bases and the expert offsets / row blocks (scan_and_blocks);
// moe_align_assign_kernel then places every entry. part[c * n_local + e]
// holds chunk c's count, then its base row. `counter` starts and ends zero.
constexpr int kAlignChunk = 2048;
constexpr int kAlignMTThreads = 512;

__global__ void __launch_bounds__(kAlignMTThreads)
    moe_align_hist_kernel(MoeAlignArgs a, int* part, int* counter) {
  __shared__ int cnt[kMaxLocalExperts];
  __shared__ int off[kMaxLocalExperts + 1];
  __shared__ int boff[kMaxLocalExperts + 1];
  __shared__ int s_last;
  pdl_wait();
  pdl_trigger();
  const int n = a.T * a.top_k;
  const int c = blockIdx.x;
  const int i0 = c * kAlignChunk, i1 = min(n, i0 + kAlignChunk);
  for (int e = threadIdx.x; e < a.n_local; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
    const int e = a.ids[i] - a.expert_start;
    int slot = -1;
    if (e >= 0 && e < a.n_local) slot = atomicAdd(&cnt[e], 1);
    a.inv[i] = slot;  // provisional: slot within (chunk, expert)
  }
  __syncthreads();
  for (int e = threadIdx.x; e < a.n_local; e += blockDim.x) part[c * a.n_local + e] = cnt[e];
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = (atomicAdd(counter, 1) == (int)gridDim.x - 1);
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const int C = gridDim.x;
  for (int e = threadIdx.x; e < a.n_local; e += blockDim.x) {
    int run = 0;
    for (int cc = 0; cc < C; ++cc) {
      const int v = __ldcg(part + cc * a.n_local + e);
      part[cc * a.n_local + e] = run;  // exclusive prefix within the expert
      run += v;
    }
    cnt[e] = run;
  }
  __syncthreads();
  scan_and_blocks(cnt, off, boff, a);
  for (int e = threadIdx.x; e < a.n_local; e += blockDim.x)
    for (int cc = 0; cc < C; ++cc) part[cc * a.n_local + e] += off[e];
  if (threadIdx.x == 0) *counter = 0;
}

__global__ void __launch_bounds__(kAlignMTThreads)
    moe_align_assign_kernel(MoeAlignArgs a, const int* part) {
  pdl_wait();
  pdl_trigger();
  const int n = a.T * a.top_k;
  const int c = blockIdx.x;
  const int i0 = c * kAlignChunk, i1 = min(n, i0 + kAlignChunk);
  for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
    const int slot = a.inv[i];
    if (slot < 0) continue;
    const int e = a.ids[i] - a.expert_start;
    const int row = part[c * a.n_local + e] + slot;
    a.inv[i] = row;
    a.row_token[row] = i / a.top_k;
    a.row_weight[row] = a.weights[i];
  }
}

int launch_moe_align_mt(const MoeAlignArgs& a, int* part, int* counter, cudaStream_t s) {
  if (a.n_local > kMaxLocalExperts || a.block_n <= 0) return 1;
  const int n = a.T * a.top_k;
  if (n == 0) return 0;
  const int C = (n + kAlignChunk - 1) / kAlignChunk;
  int e = (int)launch_k(moe_align_hist_kernel, dim3(C), dim3(kAlignMTThreads), 0, s, a, part,
                        counter);
  if (e) return e;
  return (int)launch_k(moe_align_assign_kernel, dim3(C), dim3(kAlignMTThreads), 0, s, a,
                       (const int*)part);
}

// Router softmax/top-k for all T tokens (one warp per token) followed by the
// routing of moe_align_kernel, in one single-CTA launch (T * top_k <= 4096).
constexpr int kRouteMaxEntries = 4096;

__global__ void __launch_bounds__(kAlignThreads) moe_route_kernel(RouterArgs r, MoeAlignArgs a) {
  __shared__ int cnt[kMaxLocalExperts];
  __shared__ int off[kMaxLocalExperts + 1];
  __shared__ int boff[kMaxLocalExperts + 1];
  __shared__ int32_t s_ids[kRouteMaxEntries];
  __shared__ float s_w[kRouteMaxEntries];
  pdl_wait();
  pdl_trigger();
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  for (int t = warp; t < r.T; t += blockDim.x / 32)
    topk_token(r.logits + (size_t)t * r.ld_logits, r.E, r.top_k, r.renorm, lane,
               s_ids + t * r.top_k, s_w + t * r.top_k);
  __syncthreads();
  const int n = r.T * r.top_k;
  if (r.ids != nullptr)
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      r.ids[i] = s_ids[i];
      r.weights[i] = s_w[i];
    }
  align_body(s_ids, s_w, a, cnt, off, boff);
}

int launch_moe_route(const RouterArgs& r, const MoeAlignArgs& a, cudaStream_t s) {
  if (r.T * r.top_k > kRouteMaxEntries || r.E > 256 || r.top_k > 16 ||
      a.n_local > kMaxLocalExperts || a.block_n <= 0)
    return 1;
  return (int)launch_k(moe_route_kernel, dim3(1), dim3(kAlignThreads), 0, s, r, a);
}

// ------------------------------------------- fused MoE gate (decode) ---
// Post-attention RMSNorm + router logits + softmax/top-k/renormalise +
// routing in one launch for small token counts. CTA (tg, eg) takes the
// token group tg (kGateTok tokens) and the NTC x 8 experts of group eg:
//   1. it normalises the group's tokens into a shared-memory tile (same
//      roundings as sum_rmsnorm_kernel; group 0 also stores xn for the expert
//      GEMMs);
//   2. router logits on the tensor cores: m16n8k16 tiles (16 tokens x 8
//      experts), the CTA's 8 warps splitting the NTC tiles' K range, fp32
//      accumulation, the warps' partial tiles summed in a fixed order, one
//      bf16 rounding. Within each 32-wide chunk of H the k order is permuted
//      so that a lane's A and B fragments of two k16 steps are 8 contiguous
//      values: one 16-byte load per token row (shared) and per expert row
//      (global). A and B are permuted alike and the summation order is
//      fixed, so results are deterministic;
//   3. the last of a token group's CTAs (per-group counter) runs its
//      softmax / top-k / renormalise, a warp per token;
//   4. the last group to finish (global counter) runs the routing of
//      moe_align_kernel, with ids, weights and slots in shared memory.
// Counters are reset by the CTAs that consume them. The CTAs are few and
// short, so the gate also runs well on the handful of SMs another stream's
// GEMMs leave free. Up to kGateTokMaxT tokens the per-token kernel below runs
// instead (it finishes sooner there; phase stamps come from this kernel only).
constexpr int kGateThreads = 256;
constexpr int kGateTok = 16;
constexpr int kGateMaxEntries = 2048;

__host__ __device__ constexpr int gate_row_bytes(int H) { return H * 2 + 64; }  // padded row

static int moe_gate_smem_bytes(int H) {
  const int tile = kGateTok * gate_row_bytes(H);
  const int routing = kGateMaxEntries * 12;
  return tile > routing ? tile : routing;
}

template <int H, int NTC>  // hidden size; n-tiles (8 experts each) per CTA
__global__ void __launch_bounds__(kGateThreads) moe_gate_kernel(MoeGateArgs g, MoeAlignArgs a) {
  constexpr int RB = gate_row_bytes(H);
  constexpr int WPT = 8 / NTC;              // warps per n-tile
  constexpr int KW = H / WPT;               // K range of one warp
  constexpr int CH = KW / 32;               // 32-wide chunks per warp
  constexpr int PB = CH < 8 ? CH : 8;       // chunks loaded per batch
  static_assert(KW % 32 == 0, "K range per warp must be whole 32-wide chunks");
  extern __shared__ __align__(16) uint8_t gsm[];
  __shared__ __align__(16) float red[8][32][4];                  // partial C fragments
  __shared__ __nv_bfloat16 lg_s[kGateTok * 256];                 // a group's logits
  __shared__ int cnt[kMaxLocalExperts];
  __shared__ int off[kMaxLocalExperts + 1];
  __shared__ int boff[kMaxLocalExperts + 1];
  __shared__ int s_flag;
  const int E = g.E;
  const int n_eg = E / (8 * NTC);
  const int tg = blockIdx.x / n_eg, eg = blockIdx.x % n_eg;
  const int n_groups = (g.T + kGateTok - 1) / kGateTok;
  const int t0 = tg * kGateTok;
  const int nt = min(kGateTok, g.T - t0);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int r = lane >> 2, q = lane & 3;  // fragment row / k-quad
  const int ntile = warp / WPT;            // this warp's n-tile within the CTA
  const int kbase = (warp % WPT) * KW;     // and its K range
  const int e0 = (eg * NTC + ntile) * 8;   // first expert of the n-tile

  // static weights first (before waiting on the previous kernel): this
  // lane's B fragments of the first PB chunks of its K range and its slice
  // of the norm weight
  constexpr int VPL = H / 256;  // 16-byte vectors per lane and row
  const __nv_bfloat16* brow = g.w_router + (size_t)(e0 + r) * H + kbase + q * 8;
  uint4 bv[PB], nwv[VPL];
#pragma unroll
  for (int c = 0; c < PB; ++c) bv[c] = *reinterpret_cast<const uint4*>(brow + c * 32);
#pragma unroll
  for (int c = 0; c < VPL; ++c)
    nwv[c] = *reinterpret_cast<const uint4*>(g.norm_w + (c * 32 + lane) * 8);
  // phase stamps (diagnostics): [0] start, [1] inputs ready, [2] normed,
  // [3] logits of CTA 0, [4] latest logits of any CTA, [5] top-k of token
  // group 0, [6] routing start, [7] routing end
  const bool stamp0 = g.stamps != nullptr && blockIdx.x == 0 && threadIdx.x == 0;
  if (stamp0) g.stamps[0] = globaltimer_ns();
  pdl_wait();
  pdl_trigger();
  block_wait(g.wait, 140);
  if (stamp0) g.stamps[1] = globaltimer_ns();

  // 1. RMSNorm: warp w takes tokens w and w + 8 of the group (both rows
  //    requested at once); rows past the batch are zero (their logits are
  //    never used)
  {
    constexpr int NR = kGateTok / 8;  // rows per warp
    uint4 hv[NR][VPL];
#pragma unroll
    for (int i = 0; i < NR; ++i) {
      const int tt = warp + 8 * i;
#pragma unroll
      for (int c = 0; c < VPL; ++c)
        hv[i][c] = tt < nt ? *reinterpret_cast<const uint4*>(g.h + (size_t)(t0 + tt) * g.ld_h +
                                                             (c * 32 + lane) * 8)
                           : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int i = 0; i < NR; ++i) {
      const int tt = warp + 8 * i;
      float ss = 0.f;
#pragma unroll
      for (int c = 0; c < VPL; ++c) {
        const uint32_t* pv = &hv[i][c].x;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float x0, x1;
          unpack_bf16x2(pv[e], x0, x1);
          ss += x0 * x0 + x1 * x1;
        }
      }
      ss = warp_sum(ss);
      const float rstd = rsqrtf(ss / (float)H + g.eps);
      uint8_t* dst = gsm + tt * RB;
#pragma unroll
      for (int c = 0; c < VPL; ++c) {
        const int col = (c * 32 + lane) * 8;
        const uint32_t* pv = &hv[i][c].x;
        const uint32_t* pw = &nwv[c].x;
        uint4 o;
        uint32_t* po = &o.x;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float x0, x1, w0, w1;
          unpack_bf16x2(pv[e], x0, x1);
          unpack_bf16x2(pw[e], w0, w1);
          po[e] = pack_bf16x2(w0 * round_bf16(x0 * rstd), w1 * round_bf16(x1 * rstd));
        }
        *reinterpret_cast<uint4*>(dst + col * 2) = o;  // zero rows stay zero
        if (eg == 0 && tt < nt) *reinterpret_cast<uint4*>(g.xn + (size_t)(t0 + tt) * H + col) = o;
      }
    }
  }
  __syncthreads();
  if (stamp0) g.stamps[2] = globaltimer_ns();

  // 2. router logits on the tensor cores
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  {
    const uint8_t* a_lo = gsm + r * RB + (kbase + q * 8) * 2;
    const uint8_t* a_hi = gsm + (r + 8) * RB + (kbase + q * 8) * 2;
#pragma unroll 1
    for (int c0 = 0; c0 < CH; c0 += PB) {
      if (c0 > 0) {
#pragma unroll
        for (int c = 0; c < PB; ++c)
          bv[c] = *reinterpret_cast<const uint4*>(brow + (c0 + c) * 32);
      }
#pragma unroll
      for (int c = 0; c < PB; ++c) {
        const uint4 alo = *reinterpret_cast<const uint4*>(a_lo + (c0 + c) * 64);
        const uint4 ahi = *reinterpret_cast<const uint4*>(a_hi + (c0 + c) * 64);
        mma_16816_bf16(acc, alo.x, ahi.x, alo.y, ahi.y, bv[c].x, bv[c].y);
        mma_16816_bf16(acc, alo.z, ahi.z, alo.w, ahi.w, bv[c].z, bv[c].w);
      }
    }
  }
  *reinterpret_cast<float4*>(&red[warp][lane][0]) = make_float4(acc[0], acc[1], acc[2], acc[3]);
  __syncthreads();
  if (warp % WPT == 0) {
    // the n-tile's first warp sums its WPT warps' partial tiles in warp order
    float sum[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int w = 0; w < WPT; ++w) {
      const float4 v = *reinterpret_cast<const float4*>(&red[warp + w][lane][0]);
      sum[0] += v.x;
      sum[1] += v.y;
      sum[2] += v.z;
      sum[3] += v.w;
    }
    // C fragment: rows (tokens) r and r + 8, columns (experts) 2q and 2q + 1
    const int e = e0 + 2 * q;
    if (r < nt) {
      g.logits[(size_t)(t0 + r) * E + e] = __float2bfloat16_rn(sum[0]);
      g.logits[(size_t)(t0 + r) * E + e + 1] = __float2bfloat16_rn(sum[1]);
    }
    if (r + 8 < nt) {
      g.logits[(size_t)(t0 + r + 8) * E + e] = __float2bfloat16_rn(sum[2]);
      g.logits[(size_t)(t0 + r + 8) * E + e + 1] = __float2bfloat16_rn(sum[3]);
    }
  }

  // 3. the token group's last CTA: softmax / top-k / renormalise, a warp per token
  __threadfence();
  __syncthreads();
  if (g.stamps != nullptr && threadIdx.x == 0) {
    const unsigned long long now = globaltimer_ns();
    if (blockIdx.x == 0) g.stamps[3] = now;
    atomicMax(&g.stamps[4], now);
  }
  if (threadIdx.x == 0) s_flag = (atomicAdd(&g.tok_cnt[tg], 1) == n_eg - 1);
  __syncthreads();
  if (!s_flag) return;
  __threadfence();
  for (int i = threadIdx.x; i < nt * E; i += kGateThreads)
    lg_s[i] = __ushort_as_bfloat16(__ldcg(reinterpret_cast<const unsigned short*>(g.logits) +
                                          (size_t)t0 * E + i));
  __syncthreads();
  {
    // half-warp h takes token h of the group: all 16 ranked at once
    const int tt = threadIdx.x / 16;
    const bool mine = tt < nt;
    topk_halfwarp(lg_s + (mine ? tt : 0) * E, E, g.top_k, g.renorm, lane & 15, mine,
                  g.ids + (size_t)(t0 + tt) * g.top_k, g.weights + (size_t)(t0 + tt) * g.top_k);
  }
  if (threadIdx.x == 0) g.tok_cnt[tg] = 0;
  __threadfence();
  __syncthreads();
  if (g.stamps != nullptr && threadIdx.x == 0 && tg == 0) g.stamps[5] = globaltimer_ns();
  if (threadIdx.x == 0) s_flag = (atomicAdd(g.done_cnt, 1) == n_groups - 1);
  __syncthreads();
  if (!s_flag) return;

  // 4. the last group: routing over all T tokens (ids, weights and the
  //    provisional slots stay in shared memory)
  __threadfence();
  if (g.stamps != nullptr && threadIdx.x == 0) g.stamps[6] = globaltimer_ns();
  int32_t* s_ids = reinterpret_cast<int32_t*>(gsm);
  float* s_w = reinterpret_cast<float*>(gsm + kGateMaxEntries * 4);
  int* s_slot = reinterpret_cast<int*>(gsm + kGateMaxEntries * 8);
  const int n = g.T * g.top_k;
  for (int e = threadIdx.x; e < a.n_local; e += kGateThreads) cnt[e] = 0;
  for (int i = threadIdx.x; i < n; i += kGateThreads) {
    s_ids[i] = __ldcg(g.ids + i);
    s_w[i] = __ldcg(g.weights + i);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += kGateThreads) {
    const int e = s_ids[i] - a.expert_start;
    s_slot[i] = (e >= 0 && e < a.n_local) ? atomicAdd(&cnt[e], 1) : -1;
  }
  __syncthreads();
  scan_and_blocks(cnt, off, boff, a);
  for (int i = threadIdx.x; i < n; i += kGateThreads) {
    const int slot = s_slot[i];
    int row = -1;
    if (slot >= 0) {
      row = off[s_ids[i] - a.expert_start] + slot;
      a.row_token[row] = i / a.top_k;
      a.row_weight[row] = s_w[i];
    }
    a.inv[i] = row;
  }
  if (threadIdx.x == 0) *g.done_cnt = 0;
  if (g.stamps != nullptr) {
    __syncthreads();
    if (threadIdx.x == 0) g.stamps[7] = globaltimer_ns();
  }
}

// n-tiles per CTA: enough CTAs (token groups x expert groups, about 128) to
// spread the router reads, at most 8 tiles (one per warp)
static int gate_ntc(int T, int E) {
  const int n_tg = (T + kGateTok - 1) / kGateTok;
  int ntc = 1;
  while (ntc < 8 && (E / (8 * ntc)) % 2 == 0 && n_tg * (E / (8 * ntc)) > 128) ntc *= 2;
  return ntc;
}

template <int H, int NTC>
static int gate_launch(const MoeGateArgs& g, const MoeAlignArgs& a, cudaStream_t s) {
  const int smem = moe_gate_smem_bytes(H);
  const cudaError_t e =
      set_max_dynamic_smem(reinterpret_cast<const void*>(moe_gate_kernel<H, NTC>), smem);
  if (e != cudaSuccess) return (int)e;
  const dim3 grid(((g.T + kGateTok - 1) / kGateTok) * (g.E / (8 * NTC))), block(kGateThreads);
  return (int)launch_k(moe_gate_kernel<H, NTC>, grid, block, smem, s, g, a);
}

template <int H>
static int gate_launch_h(const MoeGateArgs& g, const MoeAlignArgs& a, cudaStream_t s) {
  switch (gate_ntc(g.T, g.E)) {
    case 1: return gate_launch<H, 1>(g, a, s);
    case 2: return gate_launch<H, 2>(g, a, s);
    case 4: return gate_launch<H, 4>(g, a, s);
    default: return gate_launch<H, 8>(g, a, s);
  }
}

// ------------------------------------- fused MoE gate, per-token CTAs ---
// The gate for the smallest batches (up to kGateTokMaxT tokens), where one
// CTA per (token, expert group) finishes sooner than the tiled kernel below:
// CTA (t, g) normalises token t (group 0 stores xn) and computes the router
// logits of experts [g * E/G, (g+1) * E/G) with CUDA-core dot products (fp32
// accumulation, one bf16 rounding); the last of a token's G CTAs runs its
// top-k; the last token runs the routing of moe_align_kernel.
constexpr int kGateTokMaxT = 32;
constexpr int kGateTokMaxH = 4096;

template <int kVec>  // router vectors per lane = H / 256
__global__ void __launch_bounds__(kGateThreads) moe_gate_token_kernel(MoeGateArgs g, MoeAlignArgs a) {
  __shared__ float xn_s[kGateTokMaxH];
  __shared__ float red[kGateThreads / 32];
  __shared__ __nv_bfloat16 lg_s[256];
  __shared__ int cnt[kMaxLocalExperts];
  __shared__ int off[kMaxLocalExperts + 1];
  __shared__ int boff[kMaxLocalExperts + 1];
  __shared__ int32_t s_ids[kGateMaxEntries];
  __shared__ float s_w[kGateMaxEntries];
  __shared__ int s_flag;
  const int t = blockIdx.x / g.G;
  const int grp = blockIdx.x % g.G;
  const int H = g.H;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  constexpr int kChunks = (kVec + kGateThreads / 32 - 1) / (kGateThreads / 32);
  // Static weights first, before waiting on the previous kernel: this warp's
  // first router row and this thread's slice of the norm weight.
  const int per_grp = g.E / g.G;
  uint4 wv0[kVec];
#pragma unroll
  for (int c = 0; c < kVec; ++c) {
    const int col = (c * 32 + lane) * 8;
    wv0[c] = (warp < per_grp && col < H)
                 ? *reinterpret_cast<const uint4*>(g.w_router +
                                                   (size_t)(grp * per_grp + warp) * H + col)
                 : make_uint4(0, 0, 0, 0);
  }
  float nwt[kChunks][8];
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    const int col = (c * kGateThreads + threadIdx.x) * 8;
    if (col < H) load8(g.norm_w + col, nwt[c]);
  }
  pdl_wait();
  pdl_trigger();
  block_wait(g.wait, 140);

  // 1. RMSNorm of token t
  float xv[kChunks][8];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    const int col = (c * kGateThreads + threadIdx.x) * 8;
    if (col < H) {
      load8(g.h + (size_t)t * g.ld_h + col, xv[c]);
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += xv[c][i] * xv[c][i];
    }
  }
  const float tot = block_sum<kGateThreads>(ss, red);
  const float rstd = rsqrtf(tot / (float)H + g.eps);
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    const int col = (c * kGateThreads + threadIdx.x) * 8;
    if (col < H) {
      float y[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        y[i] = round_bf16(nwt[c][i] * round_bf16(xv[c][i] * rstd));
        xn_s[col + i] = y[i];
      }
      if (grp == 0) store8(g.xn + (size_t)t * H + col, y);
    }
  }
  __syncthreads();

  // 2. router logits of this CTA's experts: warp w takes experts w, w + 8, ...
  for (int j = warp; j < per_grp; j += kGateThreads / 32) {
    const int e = grp * per_grp + j;
    const __nv_bfloat16* wr = g.w_router + (size_t)e * H;
    // the row's vectors (H <= 4096: at most 16 per lane) are all requested
    // before the dot product (the first row was requested before the wait)
    uint4 wv[kVec];
#pragma unroll
    for (int c = 0; c < kVec; ++c) {
      const int col = (c * 32 + lane) * 8;
      wv[c] = j == warp ? wv0[c]
                        : (col < H ? *reinterpret_cast<const uint4*>(wr + col)
                                   : make_uint4(0, 0, 0, 0));
    }
    float acc = 0.f;
#pragma unroll
    for (int c = 0; c < kVec; ++c) {
      const int col = (c * 32 + lane) * 8;
      if (col >= H) break;
      const uint32_t* pw = &wv[c].x;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float w0, w1;
        unpack_bf16x2(pw[i], w0, w1);
        acc += w0 * xn_s[col + 2 * i];
        acc += w1 * xn_s[col + 2 * i + 1];
      }
    }
    acc = warp_sum(acc);
    if (lane == 0) g.logits[(size_t)t * g.E + e] = __float2bfloat16_rn(acc);
  }

  // 3. the token's last CTA: softmax / top-k / renormalise
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_flag = (atomicAdd(&g.tok_cnt[t], 1) == g.G - 1);
  __syncthreads();
  if (!s_flag) return;
  __threadfence();
  for (int e = threadIdx.x; e < g.E; e += kGateThreads)
    lg_s[e] = __ushort_as_bfloat16(__ldcg(reinterpret_cast<const unsigned short*>(g.logits) +
                                          (size_t)t * g.E + e));
  __syncthreads();
  if (warp == 0)
    topk_token(lg_s, g.E, g.top_k, g.renorm, lane, g.ids + (size_t)t * g.top_k,
               g.weights + (size_t)t * g.top_k);
  if (threadIdx.x == 0) g.tok_cnt[t] = 0;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_flag = (atomicAdd(g.done_cnt, 1) == g.T - 1);
  __syncthreads();
  if (!s_flag) return;

  // 4. the last token: routing over all T tokens
  __threadfence();
  const int n = g.T * g.top_k;
  for (int i = threadIdx.x; i < n; i += kGateThreads) {
    s_ids[i] = __ldcg(g.ids + i);
    s_w[i] = __ldcg(g.weights + i);
  }
  __syncthreads();
  align_body(s_ids, s_w, a, cnt, off, boff);
  if (threadIdx.x == 0) *g.done_cnt = 0;
}

static int launch_moe_gate_token(MoeGateArgs g, const MoeAlignArgs& a, cudaStream_t s) {
  // expert groups: enough CTAs (T * G ~ 256) to spread the router reads, at
  // least one expert per warp
  int G = 1;
  while (g.T * G < 256 && g.E % (G * 2 * 8) == 0) G *= 2;
  if (g.E % G != 0 || g.H > kGateTokMaxH || g.H % 8 != 0) return 1;
  g.G = G;
  const dim3 grid(g.T * G), block(kGateThreads);
  if (g.H <= 1024) return (int)launch_k(moe_gate_token_kernel<4>, grid, block, 0, s, g, a);
  if (g.H <= 2048) return (int)launch_k(moe_gate_token_kernel<8>, grid, block, 0, s, g, a);
  return (int)launch_k(moe_gate_token_kernel<16>, grid, block, 0, s, g, a);
}

int launch_moe_gate(const MoeGateArgs& g, const MoeAlignArgs& a, cudaStream_t s) {
  if (g.T <= 0 || g.T * g.top_k > kGateMaxEntries || g.E > 256 || g.E % 8 != 0 ||
      g.top_k > 16 || a.n_local > kMaxLocalExperts || a.block_n <= 0)
    return 1;
  if (g.T <= kGateTokMaxT && g.stamps == nullptr) return launch_moe_gate_token(g, a, s);
  if ((g.E / 8) % gate_ntc(g.T, g.E) != 0) return 1;
  switch (g.H) {
    case 1024: return gate_launch_h<1024>(g, a, s);
    case 2048: return gate_launch_h<2048>(g, a, s);
    case 4096: return gate_launch_h<4096>(g, a, s);
    default: return 1;
  }
}

// X_sorted[row] = X[row_token[row]] (16-byte vectors). Rows past num_rows idle.
// A warp per gathered row, 8 rows per CTA; each lane has up to 8 16-byte
// loads in flight before its stores.
constexpr int kGatherRowsPerCta = 8;
__global__ void __launch_bounds__(32 * kGatherRowsPerCta) moe_gather_kernel(MoeGatherArgs a) {
  pdl_wait();
  pdl_trigger();
  const int row = blockIdx.x * kGatherRowsPerCta + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (row >= *a.num_rows) return;
  const int t = a.row_token[row];
  const uint4* __restrict__ src = reinterpret_cast<const uint4*>(a.x + (size_t)t * a.ld_x);
  uint4* __restrict__ dst = reinterpret_cast<uint4*>(a.out + (size_t)row * a.H);
  const int n = a.H / 8;
  for (int i0 = 0; i0 < n; i0 += 32 * 8) {
    uint4 v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = i0 + u * 32 + lane;
      if (i < n) v[u] = src[i];
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = i0 + u * 32 + lane;
      if (i < n) dst[i] = v[u];
    }
  }
}

// out[t] = (residual ? h[t] : 0) + sum_j y[inv[t, j]]   (bf16 out, fp32 math)
// Also stored to up to kMaxPeers peer buffers; the last CTA raises the flags.
__global__ void __launch_bounds__(kNormThreads) moe_combine_kernel(MoeCombineArgs a) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  const int H = a.H;
  int rows[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) rows[j] = j < a.top_k ? a.inv[(size_t)t * a.top_k + j] : -1;
  int seg = -1;
  for (int s = 0; s < a.n_peers; ++s)
    if (t >= a.seg_offsets[s] && t < a.seg_offsets[s + 1]) seg = s;
  for (int col = threadIdx.x * 8; col < H; col += kNormThreads * 8) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    // every row's vector and the residual are requested before the sums
    // (loads in flight together)
    uint4 v[16];
#pragma unroll
    for (int j = 0; j < 16; ++j)
      v[j] = rows[j] >= 0 ? *reinterpret_cast<const uint4*>(a.y + (size_t)rows[j] * H + col)
                          : make_uint4(0, 0, 0, 0);
    uint4 res = make_uint4(0, 0, 0, 0);
    if (a.residual != nullptr)
      res = *reinterpret_cast<const uint4*>(a.residual + (size_t)t * a.ld_res + col);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      if (rows[j] < 0) continue;
      const uint32_t* pv = &v[j].x;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float y0, y1;
        unpack_bf16x2(pv[e], y0, y1);
        acc[2 * e] += y0;
        acc[2 * e + 1] += y1;
      }
    }
    if (a.residual != nullptr) {
      const uint32_t* pr = &res.x;
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
    if (a.out != nullptr) *reinterpret_cast<uint4*>(a.out + (size_t)t * a.ld_out + col) = u;
    if (seg >= 0)
      *reinterpret_cast<uint4*>(a.peer_out[seg] +
                                (size_t)(t - a.seg_offsets[seg] + a.peer_row_offset) * H + col) = u;
  }
  if (a.done_counter != nullptr) {
    __syncthreads();
    if (threadIdx.x == 0) {
      fence_sys();
      const int prev = atomicAdd(a.done_counter, 1);
      if (prev == (int)gridDim.x - 1) {
        fence_sys();
        const int v = a.signal_value + (a.epoch != nullptr ? *a.epoch : 0);
        for (int p = 0; p < a.n_flags; ++p) st_release_sys(a.flags[p], v);
        *a.done_counter = 0;
      }
    }
  }
}

// --------------------------------------------------------------- argmax ---
// One CTA per row; first index of the maximum (torch.argmax semantics).
__global__ void __launch_bounds__(1024) argmax_kernel(const __nv_bfloat16* logits, int V, int ld,
                                                      int64_t* out) {
  __shared__ float sv[32];
  __shared__ int si[32];
  pdl_wait();
  pdl_trigger();
  const int row = blockIdx.x;
  const __nv_bfloat16* p = logits + (size_t)row * ld;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float v = bf16_to_f(p[i]);
    if (v > best || (v == best && i < bi)) { best = v; bi = i; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffff, best, o);
    const int oi = __shfl_xor_sync(0xffffffff, bi, o);
    if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
  }
  const int w = threadIdx.x / 32, l = threadIdx.x % 32;
  if (l == 0) { sv[w] = best; si[w] = bi; }
  __syncthreads();
  if (w == 0) {
    const int nw = blockDim.x / 32;
    best = l < nw ? sv[l] : -INFINITY;
    bi = l < nw ? si[l] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffff, best, o);
      const int oi = __shfl_xor_sync(0xffffffff, bi, o);
      if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
    }
    // a row with no comparable value (all NaN) yields 0: always a valid token id
    if (l == 0) out[row] = bi < V ? bi : 0;
  }
}

// Split argmax: CTA (c, row) reduces chunk c of the row (16-byte loads) into
// a partial (value, index) in the workspace; the last CTA of the row (per-row
// counter, reset by it) reduces the partials. Same tie and NaN rules as
// argmax_kernel: the first index of the maximum, NaN never chosen.
// Workspace (int32): counters [rows] (zero) | values [rows * n] | indices [rows * n].
constexpr int kArgmaxThreads = 256;
constexpr int kArgmaxChunk = 8192;  // elements per CTA: 4 x 16-byte loads per thread

__device__ __forceinline__ void argmax_take(float v, int i, float& best, int& bi) {
  if (v > best || (v == best && i < bi)) { best = v; bi = i; }
}

__device__ __forceinline__ void argmax_warp(float& best, int& bi) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffff, best, o);
    const int oi = __shfl_xor_sync(0xffffffff, bi, o);
    argmax_take(ov, oi, best, bi);
  }
}

__global__ void __launch_bounds__(kArgmaxThreads) argmax_split_kernel(
    const __nv_bfloat16* logits, int V, int ld, int64_t* out, int* counters, int* partials) {
  __shared__ float sv[kArgmaxThreads / 32];
  __shared__ int si[kArgmaxThreads / 32];
  __shared__ int s_last;
  pdl_wait();
  pdl_trigger();
  const int row = blockIdx.y, chunk = blockIdx.x, n = gridDim.x, rows = gridDim.y;
  const int start = chunk * kArgmaxChunk;
  const int end = min(V, start + kArgmaxChunk);
  const int vend = start + ((end - start) / 8) * 8;
  const __nv_bfloat16* p = logits + (size_t)row * ld;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = start + threadIdx.x * 8; i < vend; i += kArgmaxThreads * 8) {
    const uint4 q = __ldg(reinterpret_cast<const uint4*>(p + i));
    const uint32_t* w = &q.x;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float a, b;
      unpack_bf16x2(w[j], a, b);
      argmax_take(a, i + 2 * j, best, bi);
      argmax_take(b, i + 2 * j + 1, best, bi);
    }
  }
  for (int i = vend + threadIdx.x; i < end; i += kArgmaxThreads) argmax_take(bf16_to_f(p[i]), i, best, bi);
  argmax_warp(best, bi);
  const int wp = threadIdx.x / 32, l = threadIdx.x % 32;
  if (l == 0) { sv[wp] = best; si[wp] = bi; }
  __syncthreads();
  int* cnt = counters;
  float* pv = reinterpret_cast<float*>(partials);
  int* pi = partials + rows * n;
  if (threadIdx.x == 0) {
    for (int k = 1; k < kArgmaxThreads / 32; ++k) argmax_take(sv[k], si[k], best, bi);
    pv[row * n + chunk] = best;
    pi[row * n + chunk] = bi;
    __threadfence();
    s_last = atomicAdd(&cnt[row], 1) == n - 1;
  }
  __syncthreads();
  if (!s_last || threadIdx.x >= 32) return;
  __threadfence();
  best = -INFINITY;
  bi = 0x7fffffff;
  for (int c = l; c < n; c += 32) argmax_take(__ldcg(pv + row * n + c), __ldcg(pi + row * n + c), best, bi);
  argmax_warp(best, bi);
  if (l == 0) {
    out[row] = bi < V ? bi : 0;  // all NaN: 0, still a valid token id
    cnt[row] = 0;
  }
}

// ---------------------------------------------------------------- flags ---
__global__ void signal_flags_kernel(FlagArgs a) {
  pdl_wait();
  pdl_trigger();
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    fence_sys();
    const int v = a.value + (a.epoch != nullptr ? *a.epoch : 0);
    for (int i = 0; i < a.n; ++i) st_release_sys(a.flags[i], v);
  }
}

// Waits until every flag >= value; bounded by timeout_ns (status on expiry).
// The dependent launch is released only after the wait, so the next kernel's
// CTAs do not sit on SMs while the flags are outstanding (with several
// streams they would starve the other streams' kernels).
__global__ void wait_flags_kernel(FlagArgs a) {
  pdl_wait();
  if (threadIdx.x < a.n && blockIdx.x == 0) {
    const int v = a.value + (a.epoch != nullptr ? *a.epoch : 0);
    wait_flag_geq(a.flags[threadIdx.x], v, a.status, 100 + threadIdx.x, a.timeout_ns);
  }
  __syncthreads();
  pdl_trigger();
}

// Copies `bytes` (multiple of 16) from src to every peer buffer with 16-byte
// NVLink stores, then the last CTA raises the peers' flags (release, system
// scope). The hand-off kernel of the transfer benchmark.
__global__ void peer_copy_kernel(PeerCopyArgs a) {
  pdl_wait();
  pdl_trigger();
  const uint4* src = reinterpret_cast<const uint4*>(a.src);
  const size_t n = a.bytes / 16;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    const uint4 v = src[i];
    for (int p = 0; p < a.n_peers; ++p) reinterpret_cast<uint4*>(a.dst[p])[i] = v;
  }
  if (a.done_counter != nullptr) {
    __syncthreads();
    if (threadIdx.x == 0) {
      fence_sys();
      if (atomicAdd(a.done_counter, 1) == (int)gridDim.x - 1) {
        fence_sys();
        const int v = a.signal_value + (a.epoch != nullptr ? *a.epoch : 0);
        for (int p = 0; p < a.n_peers; ++p) st_release_sys(a.flags[p], v);
        *a.done_counter = 0;
      }
    }
  }
}

int launch_peer_copy(const PeerCopyArgs& a, int grid, cudaStream_t s) {
  if (a.bytes % 16 != 0 || a.n_peers > 8) return 1;
  return (int)launch_k(peer_copy_kernel, dim3(grid), dim3(512), 0, s, a);
}

// Increments a device counter (the step epoch) by `by`.
__global__ void add_i32_kernel(int* p, int by) {
  pdl_wait();
  pdl_trigger();
  if (threadIdx.x == 0 && blockIdx.x == 0) *p += by;
}

// ============================================================== launchers ===
// Many rows: one warp per row (8 rows per CTA), warp-shuffle reduction only;
// H = 256 * VPL, each lane owns VPL 8-wide vectors and requests all of a
// part's vectors before adding them. Same roundings as sum_rmsnorm_kernel.
template <int VPL>
__global__ void __launch_bounds__(256) sum_rmsnorm_rows_kernel(SumNormArgs a, int rows) {
  pdl_wait();
  pdl_trigger();
  block_wait(a.wait, 130);
  const int row = blockIdx.x * 8 + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (row >= rows) return;
  float xv[VPL][8];
#pragma unroll
  for (int c = 0; c < VPL; ++c)
#pragma unroll
    for (int i = 0; i < 8; ++i) xv[c][i] = 0.f;
  for (int p = 0; p < a.n_parts; ++p) {
    uint4 v[VPL];
#pragma unroll
    for (int c = 0; c < VPL; ++c)
      v[c] = *reinterpret_cast<const uint4*>(a.parts[p] + (size_t)row * a.ld_in +
                                             (c * 32 + lane) * 8);
#pragma unroll
    for (int c = 0; c < VPL; ++c) {
      const uint32_t* q = &v[c].x;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float u0, u1;
        unpack_bf16x2(q[e], u0, u1);
        xv[c][2 * e] += u0;
        xv[c][2 * e + 1] += u1;
      }
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < VPL; ++c) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      xv[c][i] = round_bf16(xv[c][i]);
      ss += xv[c][i] * xv[c][i];
    }
    if (a.x_out != nullptr) store8(a.x_out + (size_t)row * a.H + (c * 32 + lane) * 8, xv[c]);
  }
  ss = warp_sum(ss);
  const float rstd = rsqrtf(ss / (float)a.H + a.eps);
#pragma unroll
  for (int c = 0; c < VPL; ++c) {
    const int col = (c * 32 + lane) * 8;
    float w[8], y[8];
    load8(a.weight + col, w);
#pragma unroll
    for (int i = 0; i < 8; ++i) y[i] = w[i] * round_bf16(xv[c][i] * rstd);
    store8(a.y_out + (size_t)row * a.ld_out + col, y);
  }
}

int launch_sum_rmsnorm(const SumNormArgs& a, int rows, cudaStream_t s) {
  if (a.H % 8 != 0 || a.H > kNormThreads * 8 * 4 || a.n_parts < 1 || a.n_parts > kMaxParts)
    return 1;
  if (rows == 0) return 0;
  if (rows >= 256) {
    const dim3 grid((rows + 7) / 8), block(256);
    if (a.H == 1024) return (int)launch_k(sum_rmsnorm_rows_kernel<4>, grid, block, 0, s, a, rows);
    if (a.H == 2048) return (int)launch_k(sum_rmsnorm_rows_kernel<8>, grid, block, 0, s, a, rows);
    if (a.H == 4096) return (int)launch_k(sum_rmsnorm_rows_kernel<16>, grid, block, 0, s, a, rows);
  }
  return (int)launch_k(sum_rmsnorm_kernel, dim3(rows), dim3(kNormThreads), 0, s, a);
}

// D = 128 variant for many tokens: a warp takes kQKHeads consecutive heads of
// one token and lane l the rotation pairs (j, j + 64) for j = 2l, 2l + 1, so
// every load is a 4-byte vector and the loads of all its heads are issued
// before any reduction. Same roundings as qk_norm_rope_cache_kernel.
constexpr int kQKHeads = 8;

__global__ void __launch_bounds__(256) qk_norm_rope_cache_d128_kernel(QKRopeArgs a) {
  pdl_wait();
  pdl_trigger();
  const int n_heads = a.nq + 2 * a.nkv;
  const int groups = (n_heads + kQKHeads - 1) / kQKHeads;
  const int gw = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (gw >= a.T * groups) return;
  const int t = gw / groups;
  const int h0 = (gw % groups) * kQKHeads;
  constexpr int D = 128, half = 64;
  const int j = 2 * lane;
  const int start = *a.start_pos;
  const int pos = start + t % a.q_len;
  const int b = a.batch_offset + t / a.q_len;
  const __nv_bfloat16* src = a.qkv + (size_t)t * a.ld_qkv;
  uint32_t lo[kQKHeads], hi[kQKHeads];
#pragma unroll
  for (int i = 0; i < kQKHeads; ++i) {
    const int h = h0 + i;
    lo[i] = h < n_heads ? *reinterpret_cast<const uint32_t*>(src + h * D + j) : 0u;
    hi[i] = h < n_heads ? *reinterpret_cast<const uint32_t*>(src + h * D + half + j) : 0u;
  }
  const float2 cs = *reinterpret_cast<const float2*>(a.rope + (size_t)pos * D + j);
  const float2 sn = *reinterpret_cast<const float2*>(a.rope + (size_t)pos * D + half + j);
  float qw[4], kw[4];
  {
    const uint32_t q0 = *reinterpret_cast<const uint32_t*>(a.q_norm + j);
    const uint32_t q1 = *reinterpret_cast<const uint32_t*>(a.q_norm + half + j);
    const uint32_t k0 = *reinterpret_cast<const uint32_t*>(a.k_norm + j);
    const uint32_t k1 = *reinterpret_cast<const uint32_t*>(a.k_norm + half + j);
    unpack_bf16x2(q0, qw[0], qw[1]);
    unpack_bf16x2(q1, qw[2], qw[3]);
    unpack_bf16x2(k0, kw[0], kw[1]);
    unpack_bf16x2(k1, kw[2], kw[3]);
  }
  const float c[2] = {cs.x, cs.y}, sv[2] = {sn.x, sn.y};
#pragma unroll
  for (int i = 0; i < kQKHeads; ++i) {
    const int h = h0 + i;
    if (h >= n_heads) break;  // warp-uniform
    float x[4];
    unpack_bf16x2(lo[i], x[0], x[1]);
    unpack_bf16x2(hi[i], x[2], x[3]);
    __nv_bfloat16* dst;
    if (h >= a.nq + a.nkv) {  // value head: straight copy into the cache
      dst = a.v_cache + (((size_t)b * a.nkv + (h - a.nq - a.nkv)) * a.s_max + pos) * D;
      *reinterpret_cast<uint32_t*>(dst + j) = lo[i];
      *reinterpret_cast<uint32_t*>(dst + half + j) = hi[i];
      continue;
    }
    const bool is_q = h < a.nq;
    const float* nw = is_q ? qw : kw;
    float ss = x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3];
    ss = warp_sum(ss);
    const float rstd = rsqrtf(ss / (float)D + a.eps);
    float y[4];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const float xl = round_bf16(nw[e] * round_bf16(x[e] * rstd));
      const float xh = round_bf16(nw[2 + e] * round_bf16(x[2 + e] * rstd));
      // HF: x * cos + rotate_half(x) * sin, each product and the sum in bf16
      y[e] = round_bf16(round_bf16(xl * c[e]) + round_bf16(-xh * sv[e]));
      y[2 + e] = round_bf16(round_bf16(xh * c[e]) + round_bf16(xl * sv[e]));
    }
    dst = is_q ? a.q_out + ((size_t)t * a.nq + h) * D
               : a.k_cache + (((size_t)b * a.nkv + (h - a.nq)) * a.s_max + pos) * D;
    *reinterpret_cast<uint32_t*>(dst + j) = pack_bf16x2(y[0], y[1]);
    *reinterpret_cast<uint32_t*>(dst + half + j) = pack_bf16x2(y[2], y[3]);
  }
}

int launch_qk_norm_rope_cache(const QKRopeArgs& a, cudaStream_t s) {
  if (a.D % 64 != 0 || a.D > 128) return 1;
  const int n_heads = a.nq + 2 * a.nkv;
  const int wpb = 8;
  if (a.D == 128 && a.ld_qkv % 2 == 0) {
    const int warps = a.T * ((n_heads + kQKHeads - 1) / kQKHeads);
    if (warps == 0) return 0;
    return (int)launch_k(qk_norm_rope_cache_d128_kernel, dim3((warps + wpb - 1) / wpb),
                         dim3(wpb * 32), 0, s, a);
  }
  const int warps = a.T * n_heads;
  if (warps == 0) return 0;
  return (int)launch_k(qk_norm_rope_cache_kernel, dim3((warps + wpb - 1) / wpb), dim3(wpb * 32), 0, s, a);
}

int launch_router_topk(const RouterArgs& a, cudaStream_t s) {
  if (a.E > 256 || a.top_k > 16) return 1;
  if (a.T == 0) return 0;
  const int wpb = 8;
  return (int)launch_k(router_topk_kernel, dim3((a.T + wpb - 1) / wpb), dim3(wpb * 32), 0, s, a);
}

int launch_moe_align(const MoeAlignArgs& a, cudaStream_t s) {
  if (a.n_local > kMaxLocalExperts || a.block_n <= 0) return 1;
  return (int)launch_k(moe_align_kernel, dim3(1), dim3(kAlignThreads), 0, s, a);
}

int launch_moe_gather(const MoeGatherArgs& a, int max_rows, cudaStream_t s) {
  if (a.H % 8 != 0) return 1;
  if (max_rows == 0) return 0;
  return (int)launch_k(moe_gather_kernel,
                       dim3((max_rows + kGatherRowsPerCta - 1) / kGatherRowsPerCta),
                       dim3(32 * kGatherRowsPerCta), 0, s, a);
}

int launch_moe_combine(const MoeCombineArgs& a, int T, cudaStream_t s) {
  if (a.H % 8 != 0 || a.top_k > 16) return 1;
  if (T == 0) return 0;
  return (int)launch_k(moe_combine_kernel, dim3(T), dim3(kNormThreads), 0, s, a);
}

int argmax_partial_ints(int rows, int V) {
  return 2 * rows * ((V + kArgmaxChunk - 1) / kArgmaxChunk);
}

int launch_argmax(const __nv_bfloat16* logits, int rows, int V, int ld, int64_t* out,
                  int* counters, int* partials, cudaStream_t s) {
  if (rows == 0) return 0;
  const bool split = counters != nullptr && partials != nullptr && V > kArgmaxChunk &&
                     ld % 8 == 0 && reinterpret_cast<uintptr_t>(logits) % 16 == 0 &&
                     rows <= 65535;
  if (!split)
    return (int)launch_k(argmax_kernel, dim3(rows), dim3(1024), 0, s, logits, V, ld, out);
  const dim3 grid((V + kArgmaxChunk - 1) / kArgmaxChunk, rows);
  return (int)launch_k(argmax_split_kernel, grid, dim3(kArgmaxThreads), 0, s, logits, V, ld, out,
                       counters, partials);
}

void set_pdl_override(int v) { g_pdl_override = v; }

int launch_signal_flags(const FlagArgs& a, cudaStream_t s) {
  return (int)launch_k(signal_flags_kernel, dim3(1), dim3(32), 0, s, a);
}

int launch_wait_flags(const FlagArgs& a, cudaStream_t s) {
  if (a.n > 32) return 1;
  return (int)launch_k(wait_flags_kernel, dim3(1), dim3(32), 0, s, a);
}

int launch_add_i32(int* p, int by, cudaStream_t s) {
  return (int)launch_k(add_i32_kernel, dim3(1), dim3(32), 0, s, p, by);
}

}  // namespace afd
