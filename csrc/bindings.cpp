// PyTorch bindings of the sm_100a kernels and of the peer-memory runtime
// (CUDA IPC handles, flag signal / bounded wait). Every op launches on the
// current PyTorch CUDA stream and raises on a bad argument or launch error.

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cstdlib>
#include <string>
#include <vector>

#include "gemm_tcgen05.h"
#include "kernels.h"

namespace {

using afd::GemmLaunch;

inline cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

#define CHECK_CUDA(x) TORCH_CHECK((x).is_cuda(), #x " must be a CUDA tensor")
#define CHECK_BF16(x) TORCH_CHECK((x).scalar_type() == at::kBFloat16, #x " must be bf16")
#define CHECK_ROWMAJOR(x) TORCH_CHECK((x).stride(-1) == 1, #x " must have unit inner stride")
// Every launch goes to the current stream of the device that holds the op's
// tensors, whichever device the calling thread has current (a process may
// drive several GPUs); the previous device is restored on return.
#define DEVICE_GUARD(x)                                  \
  TORCH_CHECK((x).is_cuda(), #x " must be a CUDA tensor"); \
  const c10::cuda::CUDAGuard device_guard_((x).device())

inline void check_rc(int rc, const char* what) {
  TORCH_CHECK(rc == 0, what, " failed with code ", rc,
              rc > 4000 ? std::string(" (") + cudaGetErrorString((cudaError_t)(rc - 4000)) + ")"
                        : std::string());
}

inline __nv_bfloat16* bf(const at::Tensor& t) {
  return reinterpret_cast<__nv_bfloat16*>(t.data_ptr());
}
inline const __nv_bfloat16* cbf(const at::Tensor& t) {
  return reinterpret_cast<const __nv_bfloat16*>(t.data_ptr());
}
template <typename T>
inline T* opt_ptr(const c10::optional<at::Tensor>& t) {
  return t.has_value() && t->defined() ? reinterpret_cast<T*>(t->data_ptr()) : nullptr;
}

int g_num_sms = 0;
// Upper bound on the persistent GEMM grid (0: all SMs). Set around work that
// should leave SMs to a concurrent stream (co-located attention + FFN).
static int g_sm_cap = 0;

void set_gemm_sm_cap(int64_t cap) { g_sm_cap = (int)cap; }
// -1: launches follow AFD_PDL; 0 / 1: programmatic dependent launch off / on
void set_pdl_override(int64_t v) { afd::set_pdl_override((int)v); }

int num_sms() {
  if (g_num_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
  }
  return g_num_sms;
}

// out[rows, N] = x[rows, K] @ w^T (+ epilogue); see gemm_tcgen05.cu.
void gemm(const at::Tensor& w, const at::Tensor& x, at::Tensor& out, int64_t f_tiles,
          int64_t w_rows_per_group, int64_t up_offset, const c10::optional<at::Tensor>& blocks,
          const c10::optional<at::Tensor>& num_blocks, int64_t dense_rows,
          const c10::optional<at::Tensor>& residual, const c10::optional<at::Tensor>& row_scale,
          bool swiglu, int64_t block_n, int64_t units_hint, std::vector<int64_t> peers,
          int64_t peer_row_offset, std::vector<int64_t> flags, int64_t signal_value,
          const c10::optional<at::Tensor>& done_counter, const c10::optional<at::Tensor>& status,
          const c10::optional<at::Tensor>& epoch, int64_t k_splits,
          const c10::optional<at::Tensor>& ws, const c10::optional<at::Tensor>& tile_counters,
          const c10::optional<at::Tensor>& row_ids, bool token_major, bool stream_k) {
  DEVICE_GUARD(x);
  CHECK_CUDA(w); CHECK_CUDA(x); CHECK_CUDA(out);
  CHECK_BF16(w); CHECK_BF16(x); CHECK_BF16(out);
  CHECK_ROWMAJOR(w); CHECK_ROWMAJOR(x); CHECK_ROWMAJOR(out);
  TORCH_CHECK(peers.size() <= (size_t)afd::kMaxPeers, "too many peers");
  TORCH_CHECK(flags.size() <= (size_t)afd::kMaxPeers + 1, "too many flags");
  const int64_t K = x.size(-1);
  TORCH_CHECK(w.size(-1) == K, "K mismatch: w ", w.size(-1), " x ", K);
  GemmLaunch p{};
  afd::GemmArgs& a = p.args;
  a.K = (int)K;
  a.f_tiles = (int)f_tiles;
  a.w_rows_per_group = (int)w_rows_per_group;
  a.up_offset = (int)up_offset;
  a.blocks = opt_ptr<const int4>(blocks);
  a.num_blocks = opt_ptr<const int>(num_blocks);
  TORCH_CHECK((a.blocks == nullptr) == (a.num_blocks == nullptr), "blocks/num_blocks pairing");
  a.dense_rows = (int)dense_rows;
  a.out = bf(out);
  a.ld_out = (int)out.stride(-2);
  if (residual.has_value() && residual->defined()) {
    CHECK_BF16(*residual);
    a.residual = cbf(*residual);
    a.ld_res = (int)residual->stride(-2);
  }
  a.row_scale = opt_ptr<const float>(row_scale);
  for (size_t i = 0; i < peers.size(); ++i) a.peer_out[i] = reinterpret_cast<__nv_bfloat16*>(peers[i]);
  a.n_peers = (int)peers.size();
  a.peer_row_offset = (int)peer_row_offset;
  for (size_t i = 0; i < flags.size(); ++i) a.flags[i] = reinterpret_cast<int*>(flags[i]);
  a.n_flags = (int)flags.size();
  a.signal_value = (int)signal_value;
  a.epoch = opt_ptr<const int>(epoch);
  a.done_counter = opt_ptr<int>(done_counter);
  a.status = opt_ptr<int>(status);
  a.k_splits = (int)k_splits;
  a.row_ids = opt_ptr<const int>(row_ids);
  a.ws = opt_ptr<float>(ws);
  a.tile_counters = opt_ptr<int>(tile_counters);
  if (k_splits > 1) {
    // dense: exact tile count; grouped: the caller's bound (units_hint / k_splits)
    const int64_t tiles = a.blocks == nullptr ? ((dense_rows + block_n - 1) / block_n) * f_tiles
                                              : units_hint / k_splits;
    TORCH_CHECK(a.ws != nullptr &&
                    ws->numel() >= k_splits * tiles * block_n * 128 * (swiglu ? 2 : 1),
                "split-K workspace too small");
    TORCH_CHECK(a.tile_counters != nullptr && tile_counters->numel() >= tiles,
                "split-K tile counters too small");
  }
  if (stream_k) {
    // grouped only; two pieces per tile at most; units_hint bounds the tiles
    TORCH_CHECK(a.blocks != nullptr && k_splits <= 1 && units_hint > 0,
                "stream-K: grouped GEMM without split-K, with a tile bound");
    TORCH_CHECK(a.ws != nullptr && ws->numel() >= 2 * units_hint * block_n * 128 *
                                                      (swiglu ? 2 : 1),
                "stream-K workspace too small");
    TORCH_CHECK(a.tile_counters != nullptr && tile_counters->numel() >= units_hint,
                "stream-K tile counters too small");
    a.stream_k = 1;
  }
  p.w = w.data_ptr();
  p.w_rows_total = w.numel() / K;
  p.ld_w = w.stride(-2);
  p.x = x.data_ptr();
  p.x_rows = x.numel() / K;
  p.ld_x = x.stride(-2);
  p.swiglu = swiglu;
  p.block_n = (int)block_n;
  p.units_hint = (int)units_hint;
  p.num_sms = g_sm_cap > 0 ? std::min(num_sms(), g_sm_cap) : num_sms();
  p.token_major = token_major;
  if (a.blocks == nullptr && dense_rows == 0) return;
  check_rc(afd::gemm_swapab_launch(p, cur_stream()), "gemm_swapab");
}

// Grouped down-projection GEMM (routing weight per row, rows to y) with the
// MoE combine fused into its epilogue: combined rows (+ residual) go to `out`
// (optional) and to the peers of each token segment, then the last CTA raises
// the flags. cmb_counters: int32 [>= f_tiles], zeroed once, left zeroed.
void gemm_down_combine(const at::Tensor& w, const at::Tensor& x, at::Tensor& y, int64_t f_tiles,
                       int64_t w_rows_per_group, const at::Tensor& blocks,
                       const at::Tensor& num_blocks, const at::Tensor& row_scale,
                       int64_t block_n, int64_t units_hint, const at::Tensor& inv, int64_t T,
                       int64_t top_k, const c10::optional<at::Tensor>& residual,
                       const c10::optional<at::Tensor>& out, std::vector<int64_t> peers,
                       std::vector<int64_t> seg_offsets, int64_t peer_row_offset,
                       std::vector<int64_t> flags, int64_t signal_value,
                       const c10::optional<at::Tensor>& done_counter,
                       const c10::optional<at::Tensor>& status,
                       const c10::optional<at::Tensor>& epoch, at::Tensor& cmb_counters) {
  DEVICE_GUARD(x);
  CHECK_CUDA(w); CHECK_CUDA(x); CHECK_CUDA(y);
  CHECK_BF16(w); CHECK_BF16(x); CHECK_BF16(y);
  CHECK_ROWMAJOR(w); CHECK_ROWMAJOR(x); CHECK_ROWMAJOR(y);
  TORCH_CHECK(peers.size() <= (size_t)afd::kMaxPeers, "too many peers");
  TORCH_CHECK(flags.size() <= (size_t)afd::kMaxPeers + 1, "too many flags");
  TORCH_CHECK(seg_offsets.size() == (peers.empty() ? 0 : peers.size() + 1),
              "seg_offsets needs n_peers + 1 entries");
  TORCH_CHECK(cmb_counters.numel() >= f_tiles, "combine counters too small");
  TORCH_CHECK(top_k <= 16 && inv.numel() >= T * top_k, "combine: bad inverse map");
  const int64_t K = x.size(-1);
  TORCH_CHECK(w.size(-1) == K, "K mismatch");
  GemmLaunch p{};
  afd::GemmArgs& a = p.args;
  a.K = (int)K;
  a.f_tiles = (int)f_tiles;
  a.w_rows_per_group = (int)w_rows_per_group;
  a.blocks = reinterpret_cast<const int4*>(blocks.data_ptr<int32_t>());
  a.num_blocks = num_blocks.data_ptr<int32_t>();
  a.out = bf(y);
  a.ld_out = (int)y.stride(-2);
  a.row_scale = row_scale.data_ptr<float>();
  for (size_t i = 0; i < peers.size(); ++i) a.peer_out[i] = reinterpret_cast<__nv_bfloat16*>(peers[i]);
  a.n_peers = (int)peers.size();
  for (size_t i = 0; i < seg_offsets.size(); ++i) a.cmb_seg_offsets[i] = (int)seg_offsets[i];
  a.peer_row_offset = (int)peer_row_offset;
  for (size_t i = 0; i < flags.size(); ++i) a.flags[i] = reinterpret_cast<int*>(flags[i]);
  a.n_flags = (int)flags.size();
  a.signal_value = (int)signal_value;
  a.epoch = opt_ptr<const int>(epoch);
  a.done_counter = opt_ptr<int>(done_counter);
  a.status = opt_ptr<int>(status);
  a.k_splits = 1;
  a.cmb_inv = inv.data_ptr<int32_t>();
  a.cmb_T = (int)T;
  a.cmb_topk = (int)top_k;
  if (residual.has_value() && residual->defined()) {
    CHECK_BF16(*residual);
    TORCH_CHECK(residual->stride(-1) == 1, "residual rows must be contiguous");
    a.cmb_residual = cbf(*residual);
    a.cmb_ld_res = (int)residual->stride(-2);
  }
  if (out.has_value() && out->defined()) {
    CHECK_BF16(*out);
    TORCH_CHECK(out->stride(-1) == 1, "out rows must be contiguous");
    a.cmb_out = bf(*out);
    a.cmb_ld_out = (int)out->stride(-2);
  }
  a.cmb_counters = cmb_counters.data_ptr<int32_t>();
  p.w = w.data_ptr();
  p.w_rows_total = w.numel() / K;
  p.ld_w = w.stride(-2);
  p.x = x.data_ptr();
  p.x_rows = x.numel() / K;
  p.ld_x = x.stride(-2);
  p.swiglu = false;
  p.block_n = (int)block_n;
  p.units_hint = (int)units_hint;
  p.num_sms = g_sm_cap > 0 ? std::min(num_sms(), g_sm_cap) : num_sms();
  check_rc(afd::gemm_swapab_launch(p, cur_stream()), "gemm_down_combine");
}

// bounded flag wait folded into a consuming kernel (empty list: none)
static afd::FlagWait make_wait(const std::vector<int64_t>& flags, int64_t value,
                               const c10::optional<at::Tensor>& status, int64_t timeout_ns,
                               const c10::optional<at::Tensor>& epoch) {
  TORCH_CHECK(flags.size() <= (size_t)afd::kMaxFlagPeers, "too many wait flags");
  afd::FlagWait w{};
  for (size_t i = 0; i < flags.size(); ++i) w.flags[i] = reinterpret_cast<int*>(flags[i]);
  w.n = (int)flags.size();
  w.value = (int)value;
  w.epoch = opt_ptr<const int>(epoch);
  w.status = opt_ptr<int>(status);
  w.timeout_ns = (unsigned long long)timeout_ns;
  return w;
}

void sum_rmsnorm(std::vector<at::Tensor> parts, const at::Tensor& weight,
                 const c10::optional<at::Tensor>& x_out, at::Tensor& y_out, double eps,
                 std::vector<int64_t> wait_flags, int64_t wait_value,
                 const c10::optional<at::Tensor>& status, int64_t timeout_ns,
                 const c10::optional<at::Tensor>& epoch) {
  TORCH_CHECK(!parts.empty() && parts.size() <= (size_t)afd::kMaxParts, "1..8 parts");
  DEVICE_GUARD(parts[0]);
  afd::SumNormArgs a{};
  const int64_t H = parts[0].size(-1);
  const int64_t rows = parts[0].numel() / H;
  for (size_t i = 0; i < parts.size(); ++i) {
    CHECK_CUDA(parts[i]); CHECK_BF16(parts[i]); CHECK_ROWMAJOR(parts[i]);
    TORCH_CHECK(parts[i].stride(-2) == parts[0].stride(-2), "parts must share a row stride");
    a.parts[i] = cbf(parts[i]);
  }
  a.n_parts = (int)parts.size();
  a.ld_in = (int)(parts[0].dim() > 1 ? parts[0].stride(-2) : H);
  a.weight = cbf(weight);
  a.x_out = x_out.has_value() && x_out->defined() ? bf(*x_out) : nullptr;
  a.y_out = bf(y_out);
  a.ld_out = (int)(y_out.dim() > 1 ? y_out.stride(-2) : H);
  a.H = (int)H;
  a.eps = (float)eps;
  a.wait = make_wait(wait_flags, wait_value, status, timeout_ns, epoch);
  check_rc(afd::launch_sum_rmsnorm(a, (int)rows, cur_stream()), "sum_rmsnorm");
}

void qk_norm_rope_cache(const at::Tensor& qkv, const at::Tensor& q_norm, const at::Tensor& k_norm,
                        const at::Tensor& rope, at::Tensor& q_out, at::Tensor& k_cache,
                        at::Tensor& v_cache, const at::Tensor& start_pos, int64_t q_len,
                        int64_t batch_offset, int64_t nq, int64_t nkv, double eps) {
  DEVICE_GUARD(qkv);
  CHECK_BF16(qkv); CHECK_BF16(k_cache); CHECK_BF16(v_cache); CHECK_BF16(q_out);
  TORCH_CHECK(rope.scalar_type() == at::kFloat, "rope table must be fp32");
  TORCH_CHECK(start_pos.scalar_type() == at::kInt, "start_pos must be int32");
  afd::QKRopeArgs a{};
  a.qkv = cbf(qkv);
  a.ld_qkv = (int)qkv.stride(0);
  a.q_norm = cbf(q_norm);
  a.k_norm = cbf(k_norm);
  a.rope = rope.data_ptr<float>();
  a.q_out = bf(q_out);
  a.k_cache = bf(k_cache);
  a.v_cache = bf(v_cache);
  a.start_pos = start_pos.data_ptr<int>();
  a.T = (int)qkv.size(0);
  a.q_len = (int)q_len;
  a.batch_offset = (int)batch_offset;
  a.nq = (int)nq;
  a.nkv = (int)nkv;
  a.D = (int)k_cache.size(-1);
  a.s_max = (int)k_cache.size(-2);
  a.eps = (float)eps;
  check_rc(afd::launch_qk_norm_rope_cache(a, cur_stream()), "qk_norm_rope_cache");
}

void decode_attention(const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& v_cache,
                      at::Tensor& out, const at::Tensor& start_pos, int64_t batch_offset,
                      int64_t nsplit, const c10::optional<at::Tensor>& o_part,
                      const c10::optional<at::Tensor>& ml_part) {
  DEVICE_GUARD(q);
  afd::DecodeAttnArgs a{};
  a.q = cbf(q);
  a.k_cache = cbf(k_cache);
  a.v_cache = cbf(v_cache);
  a.out = bf(out);
  a.o_part = opt_ptr<float>(o_part);
  a.ml_part = opt_ptr<float>(ml_part);
  a.start_pos = start_pos.data_ptr<int>();
  a.batch_offset = (int)batch_offset;
  a.nq = (int)q.size(1);
  a.nkv = (int)k_cache.size(1);
  a.D = (int)q.size(2);
  a.s_max = (int)k_cache.size(2);
  check_rc(afd::launch_decode_attention(a, (int)q.size(0), (int)nsplit, cur_stream()),
           "decode_attention");
}

// q [B, nq, D] given (qkv empty), or the fused new-token step from qkv
// [B, ld] (q/k RMSNorm, RoPE, K/V append into the caches, then attention).
void decode_attention_tc(const c10::optional<at::Tensor>& q, at::Tensor& k_cache,
                         at::Tensor& v_cache, at::Tensor& out, const at::Tensor& start_pos,
                         int64_t batch_offset, int64_t nsplit,
                         const c10::optional<at::Tensor>& o_part,
                         const c10::optional<at::Tensor>& ml_part,
                         const c10::optional<at::Tensor>& counters,
                         const c10::optional<at::Tensor>& status, int64_t grid,
                         const c10::optional<at::Tensor>& qkv,
                         const c10::optional<at::Tensor>& q_norm,
                         const c10::optional<at::Tensor>& k_norm,
                         const c10::optional<at::Tensor>& rope, double eps) {
  DEVICE_GUARD(k_cache);
  CHECK_BF16(k_cache); CHECK_BF16(v_cache); CHECK_BF16(out);
  TORCH_CHECK(out.is_contiguous() && out.dim() == 3, "out must be contiguous [B, nq, D]");
  TORCH_CHECK(start_pos.scalar_type() == at::kInt, "start_pos must be int32");
  TORCH_CHECK(q.has_value() != qkv.has_value(), "give q or qkv");
  afd::DecodeTcArgs a{};
  if (q.has_value()) {
    CHECK_BF16(*q);
    TORCH_CHECK(q->is_contiguous(), "q must be contiguous");
    a.q = cbf(*q);
  } else {
    CHECK_BF16(*qkv);
    TORCH_CHECK(q_norm.has_value() && k_norm.has_value() && rope.has_value(),
                "the fused step needs q_norm, k_norm and the rope table");
    TORCH_CHECK(rope->scalar_type() == at::kFloat, "rope table must be fp32");
    TORCH_CHECK(qkv->stride(1) == 1, "qkv rows must be contiguous");
    a.qkv = cbf(*qkv);
    a.ld_qkv = (int)qkv->stride(0);
    a.q_norm = cbf(*q_norm);
    a.k_norm = cbf(*k_norm);
    a.rope = rope->data_ptr<float>();
    a.eps = (float)eps;
  }
  a.k_cache = bf(k_cache);
  a.v_cache = bf(v_cache);
  a.out = bf(out);
  a.o_part = opt_ptr<float>(o_part);
  a.ml_part = opt_ptr<float>(ml_part);
  a.counters = opt_ptr<int>(counters);
  a.status = opt_ptr<int>(status);
  a.start_pos = start_pos.data_ptr<int>();
  a.B = (int)out.size(0);
  a.batch_offset = (int)batch_offset;
  a.nq = (int)out.size(1);
  a.nkv = (int)k_cache.size(1);
  a.D = (int)out.size(2);
  a.s_max = (int)k_cache.size(2);
  a.nsplit = (int)nsplit;
  check_rc(afd::launch_decode_attention_tc(a, (int)grid, cur_stream()), "decode_attention_tc");
}

bool decode_tc_supported(int64_t nq, int64_t nkv, int64_t D) {
  return afd::decode_tc_supported((int)nq, (int)nkv, (int)D) != 0;
}

void decode_attention_fused(const at::Tensor& qkv, const at::Tensor& q_norm,
                            const at::Tensor& k_norm, const at::Tensor& rope, at::Tensor& k_cache,
                            at::Tensor& v_cache, at::Tensor& out, const at::Tensor& start_pos,
                            int64_t batch_offset, int64_t nq, double eps) {
  DEVICE_GUARD(qkv);
  CHECK_BF16(qkv); CHECK_BF16(k_cache); CHECK_BF16(v_cache); CHECK_BF16(out);
  TORCH_CHECK(rope.scalar_type() == at::kFloat, "rope table must be fp32");
  afd::FusedDecodeArgs a{};
  a.qkv = cbf(qkv);
  a.ld_qkv = (int)qkv.stride(0);
  a.q_norm = cbf(q_norm);
  a.k_norm = cbf(k_norm);
  a.rope = rope.data_ptr<float>();
  a.k_cache = bf(k_cache);
  a.v_cache = bf(v_cache);
  a.out = bf(out);
  a.start_pos = start_pos.data_ptr<int>();
  a.batch_offset = (int)batch_offset;
  a.nq = (int)nq;
  a.nkv = (int)k_cache.size(1);
  a.D = (int)k_cache.size(3);
  a.s_max = (int)k_cache.size(2);
  a.eps = (float)eps;
  check_rc(afd::launch_decode_attention_fused(a, (int)qkv.size(0), cur_stream()),
           "decode_attention_fused");
}

void prefill_attention(const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& v_cache,
                       at::Tensor& out, const at::Tensor& start_pos, int64_t q_len,
                       int64_t batch_offset, const c10::optional<at::Tensor>& key_lo,
                       const c10::optional<at::Tensor>& key_hi, int64_t variant) {
  DEVICE_GUARD(q);
  afd::PrefillAttnArgs a{};
  a.q = cbf(q);
  a.k_cache = cbf(k_cache);
  a.v_cache = cbf(v_cache);
  a.out = bf(out);
  a.start_pos = start_pos.data_ptr<int>();
  a.q_len = (int)q_len;
  a.batch_offset = (int)batch_offset;
  a.nq = (int)q.size(1);
  a.nkv = (int)k_cache.size(1);
  a.D = (int)q.size(2);
  a.s_max = (int)k_cache.size(2);
  const int B = (int)(q.size(0) / q_len);
  const bool masked = key_lo.has_value() && key_hi.has_value();
  if (masked) {
    TORCH_CHECK(key_lo->scalar_type() == at::kInt && key_hi->scalar_type() == at::kInt &&
                    key_lo->is_cuda() && key_hi->is_cuda() && key_lo->is_contiguous() &&
                    key_hi->is_contiguous() && key_lo->numel() >= batch_offset + B &&
                    key_hi->numel() >= batch_offset + B,
                "key_lo / key_hi: contiguous int32 CUDA tensors with a row per cache row");
    a.key_lo = key_lo->data_ptr<int>();
    a.key_hi = key_hi->data_ptr<int>();
  }
  // variant 0: tcgen05 kernel for head_dim 128 without a padding mask, two
  // heads per CTA when the GQA group is even; 1: tcgen05, one head per CTA;
  // 2: the mma.sync kernel (which also takes key ranges)
  TORCH_CHECK(variant >= 0 && variant <= 2, "prefill_attention: variant 0, 1 or 2");
  if (a.D == 128 && variant != 2 && !masked)
    check_rc(afd::launch_prefill_attention_tc(a, B, cur_stream(), variant == 0),
             "prefill_attention_tc");
  else
    check_rc(afd::launch_prefill_attention(a, B, cur_stream()), "prefill_attention");
}

void router_topk(const at::Tensor& logits, at::Tensor& ids, at::Tensor& weights, int64_t top_k,
                 bool renorm) {
  DEVICE_GUARD(logits);
  afd::RouterArgs a{};
  a.logits = cbf(logits);
  a.ld_logits = (int)logits.stride(0);
  a.ids = ids.data_ptr<int32_t>();
  a.weights = weights.data_ptr<float>();
  a.T = (int)logits.size(0);
  a.E = (int)logits.size(1);
  a.top_k = (int)top_k;
  a.renorm = renorm ? 1 : 0;
  check_rc(afd::launch_router_topk(a, cur_stream()), "router_topk");
}

void moe_align(const at::Tensor& ids, const at::Tensor& weights, int64_t expert_start,
               int64_t n_local, int64_t block_n, at::Tensor& inv, at::Tensor& row_token,
               at::Tensor& row_weight, at::Tensor& expert_offsets, at::Tensor& blocks,
               at::Tensor& num_blocks, at::Tensor& num_rows) {
  DEVICE_GUARD(ids);
  afd::MoeAlignArgs a{};
  a.ids = ids.data_ptr<int32_t>();
  a.weights = weights.data_ptr<float>();
  a.T = (int)ids.size(0);
  a.top_k = (int)ids.size(1);
  a.expert_start = (int)expert_start;
  a.n_local = (int)n_local;
  a.block_n = (int)block_n;
  a.inv = inv.data_ptr<int32_t>();
  a.row_token = row_token.data_ptr<int32_t>();
  a.row_weight = row_weight.data_ptr<float>();
  a.expert_offsets = expert_offsets.data_ptr<int32_t>();
  a.blocks = reinterpret_cast<int4*>(blocks.data_ptr<int32_t>());
  a.num_blocks = num_blocks.data_ptr<int32_t>();
  a.num_rows = num_rows.data_ptr<int32_t>();
  check_rc(afd::launch_moe_align(a, cur_stream()), "moe_align");
}

// multi-CTA routing (large T); part / counter are int32 scratch
void moe_align_mt(const at::Tensor& ids, const at::Tensor& weights, int64_t expert_start,
               int64_t n_local, int64_t block_n, at::Tensor& inv, at::Tensor& row_token,
               at::Tensor& row_weight, at::Tensor& expert_offsets, at::Tensor& blocks,
               at::Tensor& num_blocks, at::Tensor& num_rows, at::Tensor& part,
               at::Tensor& counter) {
  DEVICE_GUARD(ids);
  afd::MoeAlignArgs a{};
  a.ids = ids.data_ptr<int32_t>();
  a.weights = weights.data_ptr<float>();
  a.T = (int)ids.size(0);
  a.top_k = (int)ids.size(1);
  a.expert_start = (int)expert_start;
  a.n_local = (int)n_local;
  a.block_n = (int)block_n;
  a.inv = inv.data_ptr<int32_t>();
  a.row_token = row_token.data_ptr<int32_t>();
  a.row_weight = row_weight.data_ptr<float>();
  a.expert_offsets = expert_offsets.data_ptr<int32_t>();
  a.blocks = reinterpret_cast<int4*>(blocks.data_ptr<int32_t>());
  a.num_blocks = num_blocks.data_ptr<int32_t>();
  a.num_rows = num_rows.data_ptr<int32_t>();
  TORCH_CHECK(part.numel() >= ((ids.numel() + 2047) / 2048) * n_local && counter.numel() >= 1,
              "moe_align_mt: scratch too small");
  check_rc(afd::launch_moe_align_mt(a, part.data_ptr<int32_t>(), counter.data_ptr<int32_t>(),
                                    cur_stream()),
           "moe_align_mt");
}

// router softmax/top-k from logits + routing, one launch; ids / weights are
// written too (for callers that want them)
void moe_route(const at::Tensor& logits, at::Tensor& ids, at::Tensor& weights, int64_t top_k,
               bool renorm, int64_t expert_start, int64_t n_local, int64_t block_n,
               at::Tensor& inv, at::Tensor& row_token, at::Tensor& row_weight,
               at::Tensor& expert_offsets, at::Tensor& blocks, at::Tensor& num_blocks,
               at::Tensor& num_rows) {
  DEVICE_GUARD(logits);
  afd::RouterArgs r{};
  r.logits = cbf(logits);
  r.ld_logits = (int)logits.stride(0);
  r.ids = ids.data_ptr<int32_t>();
  r.weights = weights.data_ptr<float>();
  r.T = (int)logits.size(0);
  r.E = (int)logits.size(1);
  r.top_k = (int)top_k;
  r.renorm = renorm ? 1 : 0;
  afd::MoeAlignArgs a{};
  a.T = r.T;
  a.top_k = r.top_k;
  a.expert_start = (int)expert_start;
  a.n_local = (int)n_local;
  a.block_n = (int)block_n;
  a.inv = inv.data_ptr<int32_t>();
  a.row_token = row_token.data_ptr<int32_t>();
  a.row_weight = row_weight.data_ptr<float>();
  a.expert_offsets = expert_offsets.data_ptr<int32_t>();
  a.blocks = reinterpret_cast<int4*>(blocks.data_ptr<int32_t>());
  a.num_blocks = num_blocks.data_ptr<int32_t>();
  a.num_rows = num_rows.data_ptr<int32_t>();
  check_rc(afd::launch_moe_route(r, a, cur_stream()), "moe_route");
}

// post-attention RMSNorm + router + top-k + routing, one launch (decode
// sizes); counters: int32 [>= T + 1], zeroed once and left zeroed
void moe_gate(const at::Tensor& h, const at::Tensor& norm_w, const at::Tensor& w_router,
              at::Tensor& xn, at::Tensor& logits, at::Tensor& ids, at::Tensor& weights,
              at::Tensor& counters, int64_t top_k, bool renorm, double eps,
              int64_t expert_start, int64_t n_local, int64_t block_n, at::Tensor& inv,
              at::Tensor& row_token, at::Tensor& row_weight, at::Tensor& expert_offsets,
              at::Tensor& blocks, at::Tensor& num_blocks, at::Tensor& num_rows,
              std::vector<int64_t> wait_flags, int64_t wait_value,
              const c10::optional<at::Tensor>& status, int64_t timeout_ns,
              const c10::optional<at::Tensor>& epoch,
              const c10::optional<at::Tensor>& stamps) {
  DEVICE_GUARD(h);
  TORCH_CHECK(h.stride(1) == 1 && xn.is_contiguous() && logits.is_contiguous() &&
                  w_router.is_contiguous(),
              "moe_gate: contiguous rows expected");
  const int T = (int)h.size(0);
  TORCH_CHECK(counters.numel() >= T + 1, "moe_gate: counter buffer too small");
  afd::MoeGateArgs g{};
  g.h = cbf(h);
  g.ld_h = (int)h.stride(0);
  g.norm_w = cbf(norm_w);
  g.w_router = cbf(w_router);
  g.xn = bf(xn);
  g.logits = bf(logits);
  g.ids = ids.data_ptr<int32_t>();
  g.weights = weights.data_ptr<float>();
  g.tok_cnt = counters.data_ptr<int32_t>();
  g.done_cnt = counters.data_ptr<int32_t>() + T;
  g.T = T;
  g.H = (int)h.size(1);
  g.E = (int)w_router.size(0);
  g.stamps = stamps.has_value()
                 ? reinterpret_cast<unsigned long long*>(stamps->data_ptr<int64_t>())
                 : nullptr;
  g.top_k = (int)top_k;
  g.renorm = renorm ? 1 : 0;
  g.eps = (float)eps;
  g.wait = make_wait(wait_flags, wait_value, status, timeout_ns, epoch);
  afd::MoeAlignArgs a{};
  a.T = T;
  a.top_k = g.top_k;
  a.expert_start = (int)expert_start;
  a.n_local = (int)n_local;
  a.block_n = (int)block_n;
  a.inv = inv.data_ptr<int32_t>();
  a.row_token = row_token.data_ptr<int32_t>();
  a.row_weight = row_weight.data_ptr<float>();
  a.expert_offsets = expert_offsets.data_ptr<int32_t>();
  a.blocks = reinterpret_cast<int4*>(blocks.data_ptr<int32_t>());
  a.num_blocks = num_blocks.data_ptr<int32_t>();
  a.num_rows = num_rows.data_ptr<int32_t>();
  check_rc(afd::launch_moe_gate(g, a, cur_stream()), "moe_gate");
}

void moe_gather(const at::Tensor& x, const at::Tensor& row_token, const at::Tensor& num_rows,
                at::Tensor& out, int64_t max_rows) {
  DEVICE_GUARD(x);
  afd::MoeGatherArgs a{};
  a.x = cbf(x);
  a.ld_x = (int)x.stride(0);
  a.row_token = row_token.data_ptr<int32_t>();
  a.num_rows = num_rows.data_ptr<int32_t>();
  a.out = bf(out);
  a.H = (int)x.size(1);
  check_rc(afd::launch_moe_gather(a, (int)max_rows, cur_stream()), "moe_gather");
}

void moe_combine(const at::Tensor& y, const at::Tensor& inv, int64_t T, int64_t top_k,
                 const c10::optional<at::Tensor>& residual, const c10::optional<at::Tensor>& out,
                 std::vector<int64_t> peers, std::vector<int64_t> seg_offsets,
                 int64_t peer_row_offset, std::vector<int64_t> flags, int64_t signal_value,
                 const c10::optional<at::Tensor>& done_counter,
                 const c10::optional<at::Tensor>& epoch) {
  DEVICE_GUARD(y);
  TORCH_CHECK(peers.size() <= 8 && flags.size() <= (size_t)afd::kMaxFlagPeers, "too many peers");
  TORCH_CHECK(peers.empty() || seg_offsets.size() == peers.size() + 1,
              "seg_offsets needs one entry per peer plus the end");
  afd::MoeCombineArgs a{};
  a.y = cbf(y);
  a.inv = inv.data_ptr<int32_t>();
  a.H = (int)y.size(1);
  a.top_k = (int)top_k;
  if (residual.has_value() && residual->defined()) {
    a.residual = cbf(*residual);
    a.ld_res = (int)residual->stride(0);
  }
  if (out.has_value() && out->defined()) {
    a.out = bf(*out);
    a.ld_out = (int)out->stride(0);
  } else {
    a.ld_out = a.H;
  }
  for (size_t i = 0; i < peers.size(); ++i) a.peer_out[i] = reinterpret_cast<__nv_bfloat16*>(peers[i]);
  for (size_t i = 0; i < seg_offsets.size() && i < 9; ++i) a.seg_offsets[i] = (int)seg_offsets[i];
  a.n_peers = (int)peers.size();
  a.peer_row_offset = (int)peer_row_offset;
  for (size_t i = 0; i < flags.size(); ++i) a.flags[i] = reinterpret_cast<int*>(flags[i]);
  a.n_flags = (int)flags.size();
  a.signal_value = (int)signal_value;
  a.epoch = opt_ptr<const int>(epoch);
  a.done_counter = opt_ptr<int>(done_counter);
  check_rc(afd::launch_moe_combine(a, (int)T, cur_stream()), "moe_combine");
}

void argmax(const at::Tensor& logits, at::Tensor& out, const c10::optional<at::Tensor>& counters,
            const c10::optional<at::Tensor>& partials) {
  DEVICE_GUARD(logits);
  CHECK_BF16(logits);
  TORCH_CHECK(logits.stride(1) == 1, "argmax: rows must be contiguous");
  const int rows = (int)logits.size(0);
  int* c = nullptr;
  int* w = nullptr;
  if (counters.has_value() && partials.has_value()) {
    TORCH_CHECK(counters->scalar_type() == at::kInt && counters->is_cuda() &&
                    counters->is_contiguous() && counters->numel() >= rows,
                "argmax counters: contiguous zeroed int32 CUDA tensor, one per row");
    TORCH_CHECK(partials->scalar_type() == at::kInt && partials->is_cuda() &&
                    partials->is_contiguous() &&
                    partials->numel() >= afd::argmax_partial_ints(rows, (int)logits.size(1)),
                "argmax partials: contiguous int32 CUDA tensor of argmax_partial_ints ints");
    c = counters->data_ptr<int>();
    w = partials->data_ptr<int>();
  }
  check_rc(afd::launch_argmax(cbf(logits), rows, (int)logits.size(1), (int)logits.stride(0),
                              out.data_ptr<int64_t>(), c, w, cur_stream()),
           "argmax");
}

int64_t argmax_partial_ints(int64_t rows, int64_t V) {
  return afd::argmax_partial_ints((int)rows, (int)V);
}

afd::FlagArgs flag_args(const std::vector<int64_t>& flags, int64_t value,
                        const c10::optional<at::Tensor>& status, int64_t timeout_ns,
                        const c10::optional<at::Tensor>& epoch) {
  TORCH_CHECK(flags.size() <= 32, "at most 32 flags");
  afd::FlagArgs a{};
  for (size_t i = 0; i < flags.size(); ++i) a.flags[i] = reinterpret_cast<int*>(flags[i]);
  a.n = (int)flags.size();
  a.value = (int)value;
  a.epoch = opt_ptr<const int>(epoch);
  a.status = opt_ptr<int>(status);
  a.timeout_ns = (unsigned long long)timeout_ns;
  return a;
}

void signal_flags(std::vector<int64_t> flags, int64_t value,
                  const c10::optional<at::Tensor>& epoch) {
  c10::cuda::OptionalCUDAGuard device_guard_;
  if (epoch.has_value() && epoch->is_cuda()) device_guard_.set_device(epoch->device());
  check_rc(afd::launch_signal_flags(flag_args(flags, value, c10::nullopt, 0, epoch), cur_stream()),
           "signal_flags");
}

// Bounded device-side wait (never a host block): the stream stalls until all
// flags reach the target or `timeout_ns` passes, in which case the status
// word records kTimeoutPeerFlag and the stream continues.
void wait_flags(std::vector<int64_t> flags, int64_t value, const c10::optional<at::Tensor>& status,
                int64_t timeout_ns, const c10::optional<at::Tensor>& epoch) {
  c10::cuda::OptionalCUDAGuard device_guard_;
  if (status.has_value() && status->is_cuda()) device_guard_.set_device(status->device());
  else if (epoch.has_value() && epoch->is_cuda()) device_guard_.set_device(epoch->device());
  check_rc(afd::launch_wait_flags(flag_args(flags, value, status, timeout_ns, epoch), cur_stream()),
           "wait_flags");
}

void peer_copy(const at::Tensor& src, std::vector<int64_t> dst, std::vector<int64_t> flags,
               int64_t signal_value, const c10::optional<at::Tensor>& done_counter,
               const c10::optional<at::Tensor>& epoch, int64_t grid) {
  DEVICE_GUARD(src);
  TORCH_CHECK(dst.size() <= 8 && flags.size() == dst.size(), "1..8 peers with one flag each");
  afd::PeerCopyArgs a{};
  a.src = src.data_ptr();
  for (size_t i = 0; i < dst.size(); ++i) {
    a.dst[i] = reinterpret_cast<void*>(dst[i]);
    a.flags[i] = reinterpret_cast<int*>(flags[i]);
  }
  a.n_peers = (int)dst.size();
  a.bytes = (size_t)src.numel() * src.element_size();
  a.signal_value = (int)signal_value;
  a.epoch = opt_ptr<const int>(epoch);
  a.done_counter = opt_ptr<int>(done_counter);
  check_rc(afd::launch_peer_copy(a, (int)grid, cur_stream()), "peer_copy");
}

void add_i32(at::Tensor& t, int64_t by) {
  DEVICE_GUARD(t);
  check_rc(afd::launch_add_i32(t.data_ptr<int>(), (int)by, cur_stream()), "add_i32");
}

// ---------------------------------------------------------------- IPC ---
// Peer-visible buffers are separate cudaMalloc allocations (not sub-blocks of
// PyTorch's caching allocator), so the IPC handle of the tensor's base
// pointer names exactly that buffer. The tensor frees the memory when the
// last reference goes away.
at::Tensor ipc_alloc(int64_t nbytes, int64_t device) {
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, (size_t)nbytes);
  TORCH_CHECK(e == cudaSuccess, "cudaMalloc(", nbytes, "): ", cudaGetErrorString(e));
  e = cudaMemset(p, 0, (size_t)nbytes);
  TORCH_CHECK(e == cudaSuccess, "cudaMemset: ", cudaGetErrorString(e));
  auto opts = at::TensorOptions().dtype(at::kByte).device(at::kCUDA, (c10::DeviceIndex)device);
  return torch::from_blob(p, {nbytes}, [](void* q) { cudaFree(q); }, opts);
}

pybind11::bytes ipc_handle(const at::Tensor& t) {
  DEVICE_GUARD(t);
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, t.data_ptr());
  TORCH_CHECK(e == cudaSuccess, "cudaIpcGetMemHandle: ", cudaGetErrorString(e));
  return pybind11::bytes(reinterpret_cast<const char*>(&h), sizeof(h));
}

int64_t ipc_open(const std::string& handle) {
  TORCH_CHECK(handle.size() == sizeof(cudaIpcMemHandle_t), "bad IPC handle size");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle.data(), sizeof(h));
  void* p = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  TORCH_CHECK(e == cudaSuccess, "cudaIpcOpenMemHandle: ", cudaGetErrorString(e));
  return (int64_t)reinterpret_cast<uintptr_t>(p);
}

void ipc_close(int64_t ptr) { cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr)); }

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "afd_demo_b200 sm_100a kernels";
  m.def("num_sms", &num_sms);
  m.def("gemm", &gemm);
  m.def("sum_rmsnorm", &sum_rmsnorm);
  m.def("qk_norm_rope_cache", &qk_norm_rope_cache);
  m.def("decode_attention", &decode_attention);
  m.def("decode_attention_tc", &decode_attention_tc);
  m.def("decode_tc_supported", &decode_tc_supported);
  m.def("prefill_attention", &prefill_attention);
  m.def("argmax_partial_ints", &argmax_partial_ints);
  m.def("decode_attention_fused", &decode_attention_fused);
  m.def("router_topk", &router_topk);
  m.def("moe_align", &moe_align);
  m.def("moe_route", &moe_route);
  m.def("moe_gate", &moe_gate);
  m.def("set_gemm_sm_cap", &set_gemm_sm_cap);
  m.def("set_pdl_override", &set_pdl_override);
  m.def("moe_align_mt", &moe_align_mt);
  m.def("gemm_down_combine", &gemm_down_combine);
  m.def("moe_gather", &moe_gather);
  m.def("moe_combine", &moe_combine);
  m.def("argmax", &argmax);
  m.def("signal_flags", &signal_flags);
  m.def("wait_flags", &wait_flags);
  m.def("add_i32", &add_i32);
  m.def("peer_copy", &peer_copy);
  m.def("ipc_alloc", &ipc_alloc);
  m.def("ipc_handle", &ipc_handle);
  m.def("ipc_open", &ipc_open);
  m.def("ipc_close", &ipc_close);
}
