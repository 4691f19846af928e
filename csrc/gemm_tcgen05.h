// Host/device interface of the tcgen05 swap-AB GEMM (see gemm_tcgen05.cu).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace afd {

constexpr int kMaxPeers = 8;

struct GemmArgs {
  int K;                    // reduction length (multiple of 64)
  int f_tiles;              // output-feature tiles of 128 per group
  int w_rows_per_group;     // weight rows per group (2I gate_up, H down, N dense)
  int up_offset;            // SwiGLU: row offset of the up half within a group
  // row blocks: device list {row_start, n_rows, group, 0} + device count, or
  // dense mode (blocks == nullptr): ceil(dense_rows / block_n) blocks, group 0
  const int4* blocks;
  const int* num_blocks;
  int dense_rows;
  int block_n;              // filled by the launcher
  // epilogue
  __nv_bfloat16* out;
  int ld_out;
  const __nv_bfloat16* residual;   // optional, [rows, ld_res]
  int ld_res;
  const float* row_scale;          // optional, per row
  // fused peer stores + completion flag
  __nv_bfloat16* peer_out[kMaxPeers];
  int n_peers;
  int peer_row_offset;
  int* flags[kMaxPeers + 1];
  int n_flags;
  int signal_value;                // published value = *epoch + signal_value
  const int* epoch;                // optional device epoch base (CUDA-graph replays)
  int* done_counter;               // nullptr: no signal
  int* status;                     // device status word pair (may be nullptr)
  // split-K (dense, non-SwiGLU only): k_splits CTAs share a tile; split s
  // stores its partial sums to ws[s][tile][row][128] (fp32) and
  // tile_counters[tile] elects the last split, which adds the slices in split
  // order (deterministic), resets the counter and runs the epilogue. The
  // counters must start zeroed; both buffers stay private to one stream.
  int k_splits;
  float* ws;
  int* tile_counters;
  // stream-K (grouped mode, k_splits 1): every CTA takes an equal contiguous
  // range of the tiles x K/64 k-iterations; a tile cut by a range boundary
  // has two pieces, reduced like two splits (ws: 2 slices, tile_counters)
  int stream_k;
  // gathered B operand: sorted row r of a block reads row row_ids[r] of x
  // (TMA tile::gather4); nullptr: rows are contiguous in x
  const int* row_ids;
  int max_units;                   // upper bound on work units (set by the launcher)
  // fused MoE combine (grouped, non-SwiGLU, e.g. the down projection): once
  // every row block of output-feature tile ft is stored in `out`, the CTA that
  // stored the last one sums, for each of cmb_T tokens, the token's top-k rows
  // of `out` (cmb_inv[t * k + j], -1 = expert not local) in j order, adds the
  // residual, and stores the tile's 128 features to cmb_out and to the peer
  // buffer of the token's segment (peer_out[s] for cmb_seg_offsets[s] <= t <
  // cmb_seg_offsets[s + 1], row t - cmb_seg_offsets[s] + peer_row_offset,
  // row stride f_tiles * 128). In this mode peer_out/n_peers apply only to the
  // combined rows. cmb_counters[f_tiles] start zeroed and are reset after use.
  const int* cmb_inv;              // nullptr: no fused combine
  int cmb_T, cmb_topk;
  const __nv_bfloat16* cmb_residual;
  int cmb_ld_res;
  __nv_bfloat16* cmb_out;          // optional [cmb_T, cmb_ld_out]
  int cmb_ld_out;
  int cmb_seg_offsets[kMaxPeers + 1];
  int* cmb_counters;
};

struct GemmLaunch {
  GemmArgs args;
  const void* w;            // bf16 [w_rows_total, K] (row stride ld_w)
  int64_t w_rows_total;
  int64_t ld_w;
  const void* x;            // bf16 [x_rows, K] (row stride ld_x)
  int64_t x_rows;
  int64_t ld_x;
  bool swiglu;
  int block_n;              // 64 (decode-sized) or 256
  int units_hint;           // upper bound on work units (<= 0: unknown)
  int num_sms;
  // token-major kernel (gemm_tm.cu) for block_n 128 when its epilogue
  // covers the call (no split-K, gathered rows or fused combine)
  bool token_major;
};

// Returns 0 on success, a non-zero code describing the failure otherwise.
int gemm_swapab_launch(const GemmLaunch& p, cudaStream_t stream);

// Token-major variant (gemm_tm.cu): whether it takes this call, and its launcher.
bool gemm_tm_eligible(const GemmLaunch& p);
int gemm_tm_launch(const GemmLaunch& p, cudaStream_t stream);

}  // namespace afd
