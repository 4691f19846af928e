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

bool supported_layout(int group, int head_dim) {
  return (head_dim == 128 && (group == 8 || group == 4)) ||
         (head_dim == 64 && (group == 8 || group == 2));
}

}  // namespace

extern "C" int afd_decode_attention_noalloc(const void* q, const void* k_cache,
                                            const void* v_cache, void* out,
                                            const int* start_pos, int* status, int batch,
                                            int n_q_heads, int n_kv_heads, int head_dim,
                                            int max_batch, int max_seq, int batch_offset,
                                            int n_split, cudaStream_t stream) {
  // every argument is checked here, so the launcher's own argument checks
  // cannot fire and any failure after this point is a launch failure
  if (batch < 0 || n_q_heads <= 0 || n_kv_heads <= 0 || n_q_heads % n_kv_heads != 0 ||
      head_dim <= 0 || max_seq <= 0 || batch_offset < 0 || max_batch < 0 ||
      batch_offset + batch > max_batch || n_split < 1 ||
      !supported_layout(n_q_heads / n_kv_heads, head_dim))
    return AFD_NOALLOC_ERR_BAD_ARG;
  if (batch == 0) return AFD_NOALLOC_OK;  // nothing to read or write (pointers may be null)
  if (q == nullptr || k_cache == nullptr || v_cache == nullptr || out == nullptr ||
      start_pos == nullptr)
    return AFD_NOALLOC_ERR_BAD_ARG;
  const unsigned long long need = (unsigned long long)batch * n_q_heads * n_split *
                                  (unsigned long long)(head_dim + 2) * sizeof(float);
  if (n_split > 1 && need > AFD_NOALLOC_SCRATCH_BYTES) return AFD_NOALLOC_ERR_TOO_LARGE;
  // an error left by earlier, unrelated work would otherwise be reported as
  // this call's launch failure (and cleared); leave it for its owner
  if (cudaPeekAtLastError() != cudaSuccess) return AFD_NOALLOC_ERR_PENDING;
  afd::DecodeAttnArgs a{};
  a.q = reinterpret_cast<const __nv_bfloat16*>(q);
  a.k_cache = reinterpret_cast<const __nv_bfloat16*>(k_cache);
  a.v_cache = reinterpret_cast<const __nv_bfloat16*>(v_cache);
  a.out = reinterpret_cast<__nv_bfloat16*>(out);
  a.start_pos = start_pos;
  a.status = status;
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
  return afd::launch_decode_attention(a, batch, n_split, stream) == 0 ? AFD_NOALLOC_OK
                                                                       : AFD_NOALLOC_ERR_LAUNCH;
}

extern "C" const char* afd_noalloc_error_string(int code) {
  switch (code) {
    case AFD_NOALLOC_OK: return "ok";
    case AFD_NOALLOC_ERR_TOO_LARGE:
      return "request exceeds the 8 MiB static scratch: batch * n_q_heads * n_split * "
             "(head_dim + 2) * 4 bytes must fit";
    case AFD_NOALLOC_ERR_BAD_ARG:
      return "bad argument: null pointer, negative size, rows past max_batch or unsupported "
             "head layout";
    case AFD_NOALLOC_ERR_SYMBOL: return "cudaGetSymbolAddress of the scratch array failed";
    case AFD_NOALLOC_ERR_LAUNCH: return "kernel launch failed (see cudaGetLastError)";
    case AFD_NOALLOC_ERR_PENDING:
      return "an earlier CUDA error is pending on this thread (cudaPeekAtLastError); "
             "nothing was launched";
    default: return "unknown code";
  }
}
