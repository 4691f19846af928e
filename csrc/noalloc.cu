// Allocation-free decode attention entry point (see noalloc.h for who needs
// it and its limits). The split-KV partials go to a file-scope device array
// instead of caller- or library-allocated memory.

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <mutex>

#include "kernels.h"
#include "noalloc.h"

namespace {

// The scratch array: one per GPU that loads this library, alive until exit.
static __device__ __align__(256) unsigned char g_noalloc_scratch[AFD_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
void* g_scratch_addr[kMaxDevices] = {nullptr};
std::mutex g_setup_mutex;

// Device address of the scratch array on the current device. In host code
// the array's name is only a host-side stand-in, so the address must come
// from cudaGetSymbolAddress, once per device, with that device current.
int scratch_address(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return AFD_NOALLOC_ERR_SYMBOL;
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) return AFD_NOALLOC_ERR_SYMBOL;
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return AFD_NOALLOC_OK;
}

}  // namespace

extern "C" int afd_decode_attention_noalloc(const void* q, const void* k_cache,
                                            const void* v_cache, void* out,
                                            const int* start_pos, int batch, int n_q_heads,
                                            int n_kv_heads, int head_dim, int max_seq,
                                            int batch_offset, int n_split, cudaStream_t stream) {
  if (q == nullptr || k_cache == nullptr || v_cache == nullptr || out == nullptr ||
      start_pos == nullptr || batch < 0 || n_q_heads <= 0 || n_kv_heads <= 0 ||
      n_q_heads % n_kv_heads != 0 || head_dim <= 0 || max_seq <= 0 || batch_offset < 0 ||
      n_split < 1)
    return AFD_NOALLOC_ERR_BAD_ARG;
  if (batch == 0) return AFD_NOALLOC_OK;
  const unsigned long long need = (unsigned long long)batch * n_q_heads * n_split *
                                  (unsigned long long)(head_dim + 2) * sizeof(float);
  if (n_split > 1 && need > AFD_NOALLOC_SCRATCH_BYTES) return AFD_NOALLOC_ERR_TOO_LARGE;
  afd::DecodeAttnArgs a{};
  a.q = reinterpret_cast<const __nv_bfloat16*>(q);
  a.k_cache = reinterpret_cast<const __nv_bfloat16*>(k_cache);
  a.v_cache = reinterpret_cast<const __nv_bfloat16*>(v_cache);
  a.out = reinterpret_cast<__nv_bfloat16*>(out);
  a.start_pos = start_pos;
  a.batch_offset = batch_offset;
  a.nq = n_q_heads;
  a.nkv = n_kv_heads;
  a.D = head_dim;
  a.s_max = max_seq;
  if (n_split > 1) {
    void* base = nullptr;
    const int rc = scratch_address(&base);
    if (rc != AFD_NOALLOC_OK) return rc;
    a.o_part = reinterpret_cast<float*>(base);
    a.ml_part = a.o_part + (size_t)batch * n_q_heads * n_split * head_dim;
  }
  const int rc = afd::launch_decode_attention(a, batch, n_split, stream);
  if (rc == 1 || rc == 2) return AFD_NOALLOC_ERR_BAD_ARG;
  return rc == 0 ? AFD_NOALLOC_OK : AFD_NOALLOC_ERR_LAUNCH;
}

extern "C" const char* afd_noalloc_error_string(int code) {
  switch (code) {
    case AFD_NOALLOC_OK: return "ok";
    case AFD_NOALLOC_ERR_TOO_LARGE:
      return "request exceeds the 8 MiB static scratch: batch * n_q_heads * n_split * "
             "(head_dim + 2) * 4 bytes must fit";
    case AFD_NOALLOC_ERR_BAD_ARG:
      return "bad argument: null pointer, negative size or unsupported head layout";
    case AFD_NOALLOC_ERR_SYMBOL: return "cudaGetSymbolAddress of the scratch array failed";
    case AFD_NOALLOC_ERR_LAUNCH: return "kernel launch failed (see cudaGetLastError)";
    default: return "unknown code";
  }
}
