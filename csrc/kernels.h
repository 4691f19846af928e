// Argument structs and launchers of the memory-bound kernels (kernels.cu)
// and the attention kernels (attention.cu).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace afd {

constexpr int kMaxParts = 8;
constexpr int kMaxFlagPeers = 9;

// A receive folded into the consuming kernel: before reading its inputs every
// CTA waits (bounded) until each flag reaches *epoch + value. n == 0: no wait.
struct FlagWait {
  int* flags[kMaxFlagPeers];
  int n;
  int value;
  const int* epoch;
  int* status;
  unsigned long long timeout_ns;
};

struct SumNormArgs {
  const __nv_bfloat16* parts[kMaxParts];  // each [rows, ld_in]
  int n_parts;
  int ld_in;
  const __nv_bfloat16* weight;            // [H]
  __nv_bfloat16* x_out;                   // optional [rows, H]: the summed input
  __nv_bfloat16* y_out;                   // [rows, ld_out]
  int ld_out;
  int H;
  float eps;
  FlagWait wait;                          // inputs produced by peers (optional)
};

struct QKRopeArgs {
  const __nv_bfloat16* qkv;   // [T, ld_qkv]  q | k | v
  int ld_qkv;
  const __nv_bfloat16* q_norm;
  const __nv_bfloat16* k_norm;
  const float* rope;          // [max_pos, D]: cos | sin (half-dim each)
  __nv_bfloat16* q_out;       // [T, nq, D]
  __nv_bfloat16* k_cache;     // [B_max, nkv, s_max, D]
  __nv_bfloat16* v_cache;
  const int* start_pos;       // device scalar
  int T, q_len, batch_offset, nq, nkv, D, s_max;
  float eps;
};

struct DecodeAttnArgs {
  const __nv_bfloat16* q;     // [B, nq, D]
  const __nv_bfloat16* k_cache;
  const __nv_bfloat16* v_cache;
  __nv_bfloat16* out;         // [B, nq, D]
  float* o_part;              // split workspace [B, nq, nsplit, D]
  float* ml_part;             // [B, nq, nsplit, 2]
  const int* start_pos;       // position of the query token (kv_len = start + 1)
  int batch_offset, nq, nkv, D, s_max;
  // optional [2] status word: a *start_pos outside [0, s_max) is recorded as
  // kBoundsViolation and the kernel reads no key (outputs are zeros)
  int* status;
};

// Decode attention with the new token's q/k RMSNorm + RoPE + KV append folded
// in (qkv != nullptr), or over precomputed q [B, nq, D] (qkv == nullptr).
struct FusedDecodeArgs {
  const __nv_bfloat16* qkv;   // [B, ld_qkv]: q | k | v of the new token
  int ld_qkv;
  const __nv_bfloat16* q;     // used when qkv == nullptr
  const __nv_bfloat16* q_norm;
  const __nv_bfloat16* k_norm;
  const float* rope;          // [max_pos, D]
  __nv_bfloat16* k_cache;
  __nv_bfloat16* v_cache;
  __nv_bfloat16* out;         // [B, nq, D]
  const int* start_pos;
  int batch_offset, nq, nkv, D, s_max;
  float eps;
  int* status;                // optional; same out-of-range rule as DecodeAttnArgs
};

int launch_decode_attention_fused(const FusedDecodeArgs& a, int B, cudaStream_t s);

struct PrefillAttnArgs {
  const __nv_bfloat16* q;     // [B * q_len, nq, D]
  const __nv_bfloat16* k_cache;
  const __nv_bfloat16* v_cache;
  __nv_bfloat16* out;         // [B * q_len, nq, D]
  const int* start_pos;
  int q_len, batch_offset, nq, nkv, D, s_max;
  // optional per-cache-row visible key range [key_lo, key_hi) (padding masks;
  // only the mma.sync kernel reads them)
  const int* key_lo = nullptr;
  const int* key_hi = nullptr;
};

struct RouterArgs {
  const __nv_bfloat16* logits;  // [T, ld_logits]
  int ld_logits;
  int32_t* ids;                 // [T, top_k]
  float* weights;               // [T, top_k]
  int T, E, top_k, renorm;
};

struct MoeAlignArgs {
  const int32_t* ids;           // [T, top_k] global expert ids
  const float* weights;         // [T, top_k]
  int T, top_k, expert_start, n_local, block_n;
  int32_t* inv;                 // [T * top_k]: sorted row or -1
  int32_t* row_token;           // [T * top_k]
  float* row_weight;            // [T * top_k]
  int32_t* expert_offsets;      // [n_local + 1]
  int4* blocks;                 // [max blocks]
  int32_t* num_blocks;          // device scalar
  int32_t* num_rows;            // device scalar
};

// Fused post-attention RMSNorm + router + top-k + routing (moe_gate_kernel).
struct MoeGateArgs {
  const __nv_bfloat16* h;        // [T, ld_h] FFN input (attn_out + residual)
  int ld_h;
  const __nv_bfloat16* norm_w;   // [H]
  const __nv_bfloat16* w_router; // [E, H]
  __nv_bfloat16* xn;             // [T, H] normalised input (out)
  __nv_bfloat16* logits;         // [T, E] scratch
  int32_t* ids;                  // [T, top_k] (out)
  float* weights;                // [T, top_k] (out)
  int* tok_cnt;                  // [T] zeroed, self-cleaning
  int* done_cnt;                 // [1] zeroed, self-cleaning
  int T, H, E, top_k, renorm;
  int G;                         // expert groups of the per-token kernel (set by the launcher)
  unsigned long long* stamps;    // optional [8] %globaltimer stamps of the phases (diagnostics)
  float eps;
  FlagWait wait;                 // h produced by peers (optional)
};

struct MoeGatherArgs {
  const __nv_bfloat16* x;
  int ld_x;
  const int32_t* row_token;
  const int32_t* num_rows;
  __nv_bfloat16* out;           // [rows, H]
  int H;
};

struct MoeCombineArgs {
  const __nv_bfloat16* y;       // [rows, H] weighted expert outputs
  const int32_t* inv;           // [T * top_k]
  const __nv_bfloat16* residual;  // optional [T, ld_res]
  int ld_res;
  __nv_bfloat16* out;           // optional [T, ld_out]
  int ld_out;
  int H, top_k;
  // F2A stores: token t of segment s (seg_offsets[s] <= t < seg_offsets[s+1])
  // goes to row t - seg_offsets[s] + peer_row_offset of peer_out[s]
  __nv_bfloat16* peer_out[8];
  int seg_offsets[9];
  int n_peers;
  int peer_row_offset;
  int* flags[kMaxFlagPeers];
  int n_flags;
  int signal_value;
  const int* epoch;
  int* done_counter;
};

struct FlagArgs {
  int* flags[32];
  int n;
  int value;            // target = *epoch + value (epoch optional)
  const int* epoch;
  int* status;
  unsigned long long timeout_ns;
};

struct PeerCopyArgs {
  const void* src;
  void* dst[8];
  int* flags[8];
  int n_peers;
  size_t bytes;
  int signal_value;
  const int* epoch;
  int* done_counter;
};

int launch_peer_copy(const PeerCopyArgs& a, int grid, cudaStream_t s);
int launch_sum_rmsnorm(const SumNormArgs& a, int rows, cudaStream_t s);
int launch_qk_norm_rope_cache(const QKRopeArgs& a, cudaStream_t s);
int launch_router_topk(const RouterArgs& a, cudaStream_t s);
int launch_moe_align(const MoeAlignArgs& a, cudaStream_t s);
// multi-CTA routing for large T: part int32 [ceil(T*top_k / 2048) * n_local],
// counter int32 [1] zeroed (left zeroed)
int launch_moe_align_mt(const MoeAlignArgs& a, int* part, int* counter, cudaStream_t s);
// router top-k + moe_align in one launch (T * top_k <= 4096)
int launch_moe_route(const RouterArgs& r, const MoeAlignArgs& a, cudaStream_t s);
int launch_moe_gather(const MoeGatherArgs& a, int max_rows, cudaStream_t s);
// RMSNorm + router + top-k + routing in one launch (T * top_k <= 2048, H <= 4096)
int launch_moe_gate(const MoeGateArgs& g, const MoeAlignArgs& a, cudaStream_t s);
int launch_moe_combine(const MoeCombineArgs& a, int T, cudaStream_t s);
// Split argmax (several CTAs per row) when `counters` (one per row, zeroed;
// the kernel leaves them zeroed) and `partials` (argmax_partial_ints ints, no
// initial value) are given and the rows are 16-byte aligned; one CTA per row
// otherwise. The two live in separate buffers: the partials' layout depends on
// the row count, so a shared buffer would leave a smaller call's partials
// where a larger later call expects zeroed counters.
int argmax_partial_ints(int rows, int V);
int launch_argmax(const __nv_bfloat16* logits, int rows, int V, int ld, int64_t* out,
                  int* counters, int* partials, cudaStream_t s);
// Process-wide override of programmatic dependent launch for later launches:
// -1 follows AFD_PDL, 0 / 1 off / on.
void set_pdl_override(int v);
int launch_signal_flags(const FlagArgs& a, cudaStream_t s);
int launch_wait_flags(const FlagArgs& a, cudaStream_t s);
int launch_add_i32(int* p, int by, cudaStream_t s);
int launch_decode_attention(const DecodeAttnArgs& a, int B, int nsplit, cudaStream_t s);

// tcgen05/TMEM/TMA decode attention (decode_attention_tc.cu), head_dim 128,
// G = nq / nkv in {4, 8}; a persistent grid of at most `grid` CTAs.
struct DecodeTcArgs {
  const __nv_bfloat16* q;     // [B, nq, D] (unused when qkv is given)
  __nv_bfloat16* k_cache;     // [B_max, nkv, s_max, D]; written only by the fused step
  __nv_bfloat16* v_cache;
  __nv_bfloat16* out;         // [B, nq, D]
  float* o_part;              // nsplit > 1: [B * nq, nsplit, D]
  float* ml_part;             // nsplit > 1: [B * nq, nsplit, 2]
  int* counters;              // nsplit > 1: [B * nkv], zero; left zero
  const int* start_pos;       // position of the query token (kv_len = start + 1)
  int* status;                // optional [2]
  int B, batch_offset, nq, nkv, D, s_max, nsplit;
  // Fused new-token step (qkv != nullptr): the kernel applies q/k RMSNorm and
  // RoPE at *start_pos to the token's projections, appends its K and V to the
  // cache and attends; q is then unused.
  const __nv_bfloat16* qkv;   // [B, ld_qkv]: q heads | k heads | v heads
  int ld_qkv;
  const __nv_bfloat16* q_norm;
  const __nv_bfloat16* k_norm;
  const float* rope;          // [max_pos, D]: cos | sin
  float eps;
};
int decode_tc_supported(int nq, int nkv, int D);
int launch_decode_attention_tc(const DecodeTcArgs& a, int grid, cudaStream_t s);
int launch_prefill_attention(const PrefillAttnArgs& a, int B, cudaStream_t s);
// tcgen05/TMEM/TMA version (attention_tc.cu), head_dim 128
// pair_heads: two query heads of one kv group per CTA (ping-pong softmax,
// P in TMEM) when nq / nkv is even; otherwise one head per CTA
int launch_prefill_attention_tc(const PrefillAttnArgs& a, int B, cudaStream_t s,
                                bool pair_heads = true);

}  // namespace afd
