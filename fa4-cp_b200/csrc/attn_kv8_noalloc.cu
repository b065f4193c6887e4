// Allocation-free variant of fa4cp_attn_fwd_kv8 (bf16 query x e4m3 keys/values).
//
// fa4cp_attn_fwd_kv8 needs a caller-provided device workspace to hold the dequantised
// bf16 copies of K and V.  Some callers have no way to provide one at call time: an
// inference engine that has already reserved nearly all device memory for its own pools
// (a cudaMalloc there can fail or fragment the pool), a latency-sensitive caller that
// must not risk the device-wide synchronisation a cudaMalloc/cudaFree can imply, or a
// foreign-language binding that only holds the tensors it was handed and has no device
// allocator of its own.  This entry point serves them: its scratch is a fixed array
// compiled into the library, so it allocates nothing and needs only inputs and outputs.
//
// Limits and behaviour:
//  * the scratch holds at most kNoAllocScratchBytes = 32 MiB, i.e. bf16 K and V of at
//    most 8,388,608 elements each (total_k * num_heads_kv * head_dim); larger calls are
//    rejected with FA4CP_ERR_INVALID and a message saying so;
//  * every GPU that loads this part of the library keeps those 32 MiB until the process
//    exits;
//  * all calls on a device share the one array, and it keeps whatever the last call left
//    there.  Nothing in it has to start at zero: each call overwrites the part it reads
//    (the dequantised K and V) before reading it.  Calls that overlap on the GPU (two
//    streams, or two threads) race on the array and must be serialised by the caller;
//  * the first call on each device looks the array's device address up with
//    cudaGetSymbolAddress while that device is current (host code cannot use the
//    array's name as a device pointer); make that first call before any stream capture.
#include <mutex>

#include "common.cuh"

namespace fa4cp {
namespace {

constexpr int64_t kNoAllocScratchBytes = int64_t(32) << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) uint8_t g_kv8_scratch[kNoAllocScratchBytes];

std::mutex g_scratch_mutex;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_kv8_scratch on the current device (looked up once per device).
int scratch_for_current_device(void** out) {
  int dev = 0;
  FA4CP_CHECK_CUDA(cudaGetDevice(&dev));
  FA4CP_CHECK_ARG(dev >= 0 && dev < kMaxDevices, "device index %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_kv8_scratch);
    if (e != cudaSuccess || p == nullptr) {
      set_last_error("cudaGetSymbolAddress of the no-alloc scratch failed on device %d: %s", dev,
                     cudaGetErrorString(e));
      return FA4CP_ERR_CUDA;
    }
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return FA4CP_OK;
}

}  // namespace
}  // namespace fa4cp

using namespace fa4cp;

extern "C" int fa4cp_attn_fwd_kv8_noalloc(const void* q, const void* k8, const void* v8,
                                          void* out, float* lse, const int32_t* cu_q,
                                          const int32_t* cu_k, int32_t nseq,
                                          int32_t max_seqlen_q, int64_t total_q, int64_t total_k,
                                          int32_t num_heads_q, int32_t num_heads_kv,
                                          int32_t head_dim, int32_t q_dtype, int32_t pattern,
                                          int32_t causal, float softmax_scale,
                                          const float* k_descale, const float* v_descale,
                                          int32_t accumulate, void* stream) {
  FA4CP_CHECK_ARG(total_k >= 0 && num_heads_kv > 0 && head_dim > 0, "bad sizes");
  // bound the row count by division first, so that the byte count below cannot overflow
  FA4CP_CHECK_ARG(total_k <= kNoAllocScratchBytes / 4 / (int64_t(num_heads_kv) * head_dim),
                  "no-alloc kv8 attention: K/V of %lld x %d x %d elements exceed its fixed "
                  "scratch of %lld bytes (K and V of at most %lld elements each); use "
                  "fa4cp_attn_fwd_kv8 with a caller workspace",
                  (long long)total_k, num_heads_kv, head_dim, (long long)kNoAllocScratchBytes,
                  (long long)(kNoAllocScratchBytes / 4));
  const int64_t need = fa4cp_attn_kv8_workspace_bytes(total_k, num_heads_kv, head_dim);
  FA4CP_CHECK_ARG(need >= 0 && need <= kNoAllocScratchBytes,
                  "no-alloc kv8 attention needs %lld bytes of scratch for K/V of %lld x %d x %d "
                  "elements, but its fixed scratch holds %lld bytes (K and V of at most %lld "
                  "elements each); use fa4cp_attn_fwd_kv8 with a caller workspace",
                  (long long)need, (long long)total_k, num_heads_kv, head_dim,
                  (long long)kNoAllocScratchBytes, (long long)(kNoAllocScratchBytes / 4));
  void* scratch = nullptr;
  int rc = scratch_for_current_device(&scratch);
  if (rc) return rc;
  return fa4cp_attn_fwd_kv8(q, k8, v8, out, lse, cu_q, cu_k, nseq, max_seqlen_q, total_q,
                            total_k, num_heads_q, num_heads_kv, head_dim, q_dtype, pattern,
                            causal, softmax_scale, k_descale, v_descale, accumulate, scratch,
                            kNoAllocScratchBytes, stream);
}
