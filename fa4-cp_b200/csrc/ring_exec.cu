// Native ring executor: one call runs a rank's whole zig-zag ring forward.
//
// Replaces the per-step host loop of fa4_ring/ring_attention.py:121-172 (a Python loop that
// issues torch.distributed P2P ops and attention launches step by step).  Here the host
// issues every step from C++: the K/V hops as NCCL send/recv on a dedicated high-priority
// comm stream, the attention launches on the caller's stream, ordered by CUDA events only
// (the host never blocks):
//   * hop 1 waits for the caller's stream (which produced the local K/V it sends);
//   * hop s (>= 3) waits for the attention of step s-2, the last reader of the receive slot
//     it overwrites; the previous hop is ordered by the comm stream itself;
//   * the attention of step s waits for hop s.
// Hop s+1 is issued right after step s's wait, before step s's attention, so the transfer
// overlaps that attention.
//
// The NCCL communicator is this library's own (ncclCommInitRank over the cp group, NCCL
// rank = cp rank), created once per group by fa4cp_ring_comm_init from a unique id that
// the caller broadcasts.  libnccl.so.2 is opened with dlopen, so the process's already
// loaded NCCL (PyTorch's) is the one used.
#include <dlfcn.h>
#include <nccl.h>
#include <string.h>

#include <mutex>
#include <vector>

#include "common.cuh"

namespace fa4cp {
namespace {

struct NcclApi {
  ncclResult_t (*GetUniqueId)(ncclUniqueId*);
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int);
  ncclResult_t (*CommDestroy)(ncclComm_t);
  ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
  ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
  ncclResult_t (*GroupStart)();
  ncclResult_t (*GroupEnd)();
  const char* (*GetErrorString)(ncclResult_t);
  bool ok = false;
};

template <typename F>
void bind(void* h, F& fn, const char* name) {
  fn = reinterpret_cast<F>(dlsym(h, name));
}

NcclApi* nccl_api() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (h == nullptr) h = dlopen("libnccl.so.2", RTLD_NOW);
    if (h == nullptr) return;
    bind(h, api.GetUniqueId, "ncclGetUniqueId");
    bind(h, api.CommInitRank, "ncclCommInitRank");
    bind(h, api.CommDestroy, "ncclCommDestroy");
    bind(h, api.Send, "ncclSend");
    bind(h, api.Recv, "ncclRecv");
    bind(h, api.GroupStart, "ncclGroupStart");
    bind(h, api.GroupEnd, "ncclGroupEnd");
    bind(h, api.GetErrorString, "ncclGetErrorString");
    api.ok = api.GetUniqueId && api.CommInitRank && api.CommDestroy && api.Send && api.Recv &&
             api.GroupStart && api.GroupEnd && api.GetErrorString;
  });
  return api.ok ? &api : nullptr;
}

constexpr int kMaxRing = 64;

struct RingComm {
  ncclComm_t comm = nullptr;
  int nranks = 0, rank = 0, device = 0;
  cudaStream_t stream = nullptr;       // high-priority comm stream
  cudaEvent_t ev_start = nullptr;      // the caller's stream reached the call
  cudaEvent_t ev_hop[kMaxRing] = {};   // hop s landed
  cudaEvent_t ev_step[kMaxRing] = {};  // attention of step s done (its K/V slot is free)
  // optional launch timing: 2 timing events per attention launch, filled in call order
  std::vector<cudaEvent_t> tev;
  int t_used = 0;
};

void destroy_timing(RingComm* rc) {
  for (cudaEvent_t e : rc->tev)
    if (e) cudaEventDestroy(e);
  rc->tev.clear();
  rc->t_used = 0;
}

void destroy_ring(RingComm* rc) {
  destroy_timing(rc);
  if (rc->ev_start) cudaEventDestroy(rc->ev_start);
  for (int i = 0; i < kMaxRing; ++i) {
    if (rc->ev_hop[i]) cudaEventDestroy(rc->ev_hop[i]);
    if (rc->ev_step[i]) cudaEventDestroy(rc->ev_step[i]);
  }
  if (rc->stream) cudaStreamDestroy(rc->stream);
  delete rc;
}

int nccl_fail(NcclApi* api, const char* what, ncclResult_t r) {
  set_last_error("%s failed: %s", what, api->GetErrorString(r));
  return FA4CP_ERR_CUDA;
}

}  // namespace
}  // namespace fa4cp

using namespace fa4cp;

#define FA4CP_CHECK_NCCL(expr)                               \
  do {                                                       \
    ncclResult_t r_ = (expr);                                \
    if (r_ != ncclSuccess) return nccl_fail(api, #expr, r_); \
  } while (0)

extern "C" int fa4cp_ring_unique_id(uint8_t* id_out) {
  FA4CP_CHECK_ARG(id_out != nullptr, "id_out is NULL");
  NcclApi* api = nccl_api();
  FA4CP_CHECK_ARG(api != nullptr, "libnccl.so.2 could not be loaded");
  ncclUniqueId id;
  FA4CP_CHECK_NCCL(api->GetUniqueId(&id));
  memcpy(id_out, &id, sizeof(id));
  return FA4CP_OK;
}

extern "C" int fa4cp_ring_comm_init(const uint8_t* id, int32_t nranks, int32_t rank,
                                    int64_t* handle_out) {
  FA4CP_CHECK_ARG(id != nullptr && handle_out != nullptr, "null argument");
  FA4CP_CHECK_ARG(nranks >= 1 && nranks <= kMaxRing && rank >= 0 && rank < nranks,
                  "bad ring size %d / rank %d (at most %d ranks)", nranks, rank, kMaxRing);
  NcclApi* api = nccl_api();
  FA4CP_CHECK_ARG(api != nullptr, "libnccl.so.2 could not be loaded");
  RingComm* rc = new RingComm();
  rc->nranks = nranks;
  rc->rank = rank;
  cudaError_t ce = cudaGetDevice(&rc->device);
  int lo = 0, hi = 0;
  if (ce == cudaSuccess) ce = cudaDeviceGetStreamPriorityRange(&lo, &hi);
  if (ce == cudaSuccess) ce = cudaStreamCreateWithPriority(&rc->stream, cudaStreamNonBlocking, hi);
  if (ce == cudaSuccess) ce = cudaEventCreateWithFlags(&rc->ev_start, cudaEventDisableTiming);
  for (int i = 0; ce == cudaSuccess && i < nranks; ++i) {
    ce = cudaEventCreateWithFlags(&rc->ev_hop[i], cudaEventDisableTiming);
    if (ce == cudaSuccess) ce = cudaEventCreateWithFlags(&rc->ev_step[i], cudaEventDisableTiming);
  }
  if (ce != cudaSuccess) {
    set_last_error("ring stream/event creation failed: %s", cudaGetErrorString(ce));
    destroy_ring(rc);
    return FA4CP_ERR_CUDA;
  }
  if (nranks > 1) {
    ncclUniqueId uid;
    memcpy(&uid, id, sizeof(uid));
    ncclResult_t r = api->CommInitRank(&rc->comm, nranks, uid, rank);
    if (r != ncclSuccess) {
      rc->comm = nullptr;
      destroy_ring(rc);
      return nccl_fail(api, "ncclCommInitRank", r);
    }
  }
  *handle_out = reinterpret_cast<int64_t>(rc);
  return FA4CP_OK;
}

extern "C" int fa4cp_ring_comm_destroy(int64_t handle) {
  FA4CP_CHECK_ARG(handle != 0, "null ring handle");
  RingComm* rc = reinterpret_cast<RingComm*>(handle);
  NcclApi* api = nccl_api();
  cudaStreamSynchronize(rc->stream);
  if (api != nullptr && rc->comm != nullptr) api->CommDestroy(rc->comm);
  destroy_ring(rc);
  return FA4CP_OK;
}

extern "C" int fa4cp_ring_timing(int64_t handle, int32_t max_launches) {
  FA4CP_CHECK_ARG(handle != 0, "null ring handle");
  FA4CP_CHECK_ARG(max_launches >= 0 && max_launches <= (1 << 16), "bad max_launches %d",
                  max_launches);
  RingComm* rc = reinterpret_cast<RingComm*>(handle);
  destroy_timing(rc);
  rc->tev.assign(2 * size_t(max_launches), nullptr);
  for (auto& e : rc->tev) {
    cudaError_t ce = cudaEventCreate(&e);
    if (ce != cudaSuccess) {
      set_last_error("cudaEventCreate failed: %s", cudaGetErrorString(ce));
      destroy_timing(rc);
      return FA4CP_ERR_CUDA;
    }
  }
  return FA4CP_OK;
}

extern "C" int fa4cp_ring_timing_read(int64_t handle, double* total_ms, int32_t* launches) {
  FA4CP_CHECK_ARG(handle != 0 && total_ms != nullptr && launches != nullptr, "null argument");
  RingComm* rc = reinterpret_cast<RingComm*>(handle);
  double sum = 0.0;
  for (int i = 0; i < rc->t_used; ++i) {
    FA4CP_CHECK_CUDA(cudaEventSynchronize(rc->tev[2 * i + 1]));
    float ms = 0.f;
    FA4CP_CHECK_CUDA(cudaEventElapsedTime(&ms, rc->tev[2 * i], rc->tev[2 * i + 1]));
    sum += ms;
  }
  *total_ms = sum;
  *launches = rc->t_used;
  rc->t_used = 0;
  return FA4CP_OK;
}

extern "C" int fa4cp_ring_attn_fwd(int64_t handle, const void* q, const void* k, const void* v,
                                   void* kv_bufs, int64_t kv_bufs_bytes, void* out, float* lse,
                                   const int32_t* cu, int32_t nseq, int32_t max_seqlen,
                                   int64_t total, int32_t num_heads_q, int32_t num_heads_kv,
                                   int32_t head_dim, int32_t q_dtype, int32_t kv_dtype,
                                   float softmax_scale, const float* q_descale,
                                   const float* k_descales, const float* v_descales,
                                   void* workspace, int64_t workspace_bytes, void* stream) {
  FA4CP_CHECK_ARG(handle != 0, "null ring handle");
  RingComm* rc = reinterpret_cast<RingComm*>(handle);
  const int S = rc->nranks, rank = rc->rank;
  FA4CP_CHECK_ARG(q && k && v && out && lse && cu, "null tensor pointer");
  FA4CP_CHECK_ARG(total >= 0 && nseq >= 1 && max_seqlen >= 0, "bad sizes");
  FA4CP_CHECK_ARG(num_heads_kv > 0 && head_dim > 0, "bad head shape");
  const bool mixed = kv_dtype == FA4CP_DTYPE_E4M3 && q_dtype == FA4CP_DTYPE_BF16;
  FA4CP_CHECK_ARG(q_dtype == kv_dtype || mixed,
                  "q and k/v dtypes must match (or bf16 q with e4m3 k/v)");
  const int out_dtype = q_dtype == FA4CP_DTYPE_E4M3 ? FA4CP_DTYPE_BF16 : q_dtype;
  const int64_t kv_bytes = total * num_heads_kv * int64_t(head_dim) * elem_bytes(kv_dtype);
  FA4CP_CHECK_ARG(kv_bytes % 16 == 0, "K/V shard bytes must be a multiple of 16");
  FA4CP_CHECK_ARG(S == 1 || (kv_bufs != nullptr && kv_bufs_bytes >= 4 * kv_bytes),
                  "kv_bufs must hold two slots of K and V (%lld bytes)",
                  static_cast<long long>(4 * kv_bytes));
  FA4CP_CHECK_ARG(uintptr_t(kv_bufs) % 16 == 0, "kv_bufs must be 16-byte aligned");
  int dev = 0;
  FA4CP_CHECK_CUDA(cudaGetDevice(&dev));
  FA4CP_CHECK_ARG(dev == rc->device, "current device %d is not the ring's device %d", dev,
                  rc->device);
  NcclApi* api = nccl_api();
  FA4CP_CHECK_ARG(api != nullptr, "libnccl.so.2 could not be loaded");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int send_peer = (rank + 1) % S, recv_peer = (rank + S - 1) % S;
  uint8_t* bufs = static_cast<uint8_t*>(kv_bufs);
  // step s >= 1 reads slot s & 1, laid out [K | V], kv_bytes each
  auto slot_k = [&](int s) { return bufs + int64_t(s & 1) * 2 * kv_bytes; };
  auto slot_v = [&](int s) { return slot_k(s) + kv_bytes; };
  auto step_k = [&](int s) -> const void* { return s == 0 ? k : slot_k(s); };
  auto step_v = [&](int s) -> const void* { return s == 0 ? v : slot_v(s); };

  // hop s: send the K/V of step s-1 to rank+1, receive the K/V of step s from rank-1
  auto hop = [&](int s) -> int {
    if (s == 1) {
      FA4CP_CHECK_CUDA(cudaEventRecord(rc->ev_start, st));
      FA4CP_CHECK_CUDA(cudaStreamWaitEvent(rc->stream, rc->ev_start, 0));
    } else if (s >= 3) {
      FA4CP_CHECK_CUDA(cudaStreamWaitEvent(rc->stream, rc->ev_step[s - 2], 0));
    }
    FA4CP_CHECK_NCCL(api->GroupStart());
    FA4CP_CHECK_NCCL(api->Send(step_k(s - 1), size_t(kv_bytes), ncclUint8, send_peer, rc->comm,
                               rc->stream));
    FA4CP_CHECK_NCCL(api->Recv(slot_k(s), size_t(kv_bytes), ncclUint8, recv_peer, rc->comm,
                               rc->stream));
    FA4CP_CHECK_NCCL(api->Send(step_v(s - 1), size_t(kv_bytes), ncclUint8, send_peer, rc->comm,
                               rc->stream));
    FA4CP_CHECK_NCCL(api->Recv(slot_v(s), size_t(kv_bytes), ncclUint8, recv_peer, rc->comm,
                               rc->stream));
    FA4CP_CHECK_NCCL(api->GroupEnd());
    FA4CP_CHECK_CUDA(cudaEventRecord(rc->ev_hop[s], rc->stream));
    return FA4CP_OK;
  };

  int r = FA4CP_OK;
  if (S > 1 && (r = hop(1)) != FA4CP_OK) return r;  // hop 1 overlaps the local step
  for (int s = 0; s < S; ++s) {
    const int src = (rank - s + S) % S;
    const int pattern = s == 0 ? FA4CP_PATTERN_VARLEN
                               : (s > rank ? FA4CP_PATTERN_BACK_Q : FA4CP_PATTERN_FRONT_KV);
    const int q_rows = pattern == FA4CP_PATTERN_BACK_Q ? (max_seqlen + 1) / 2 : max_seqlen;
    if (s > 0) {
      FA4CP_CHECK_CUDA(cudaStreamWaitEvent(st, rc->ev_hop[s], 0));
      if (s + 1 < S && (r = hop(s + 1)) != FA4CP_OK) return r;
    }
    const float* kd = k_descales ? k_descales + int64_t(src) * num_heads_kv : nullptr;
    const float* vd = v_descales ? v_descales + int64_t(src) * num_heads_kv : nullptr;
    const bool timed = rc->t_used < int(rc->tev.size() / 2);
    if (timed) FA4CP_CHECK_CUDA(cudaEventRecord(rc->tev[2 * rc->t_used], st));
    if (mixed)
      r = fa4cp_attn_fwd_kv8(q, step_k(s), step_v(s), out, lse, cu, cu, nseq, q_rows, total,
                             total, num_heads_q, num_heads_kv, head_dim, q_dtype, pattern,
                             s == 0, softmax_scale, kd, vd, s > 0, workspace, workspace_bytes,
                             stream);
    else
      r = fa4cp_attn_fwd(q, step_k(s), step_v(s), out, lse, cu, cu, nseq, q_rows, total, total,
                         num_heads_q, num_heads_kv, head_dim, q_dtype, out_dtype, pattern, s == 0,
                         softmax_scale, q_descale, kd, vd, s > 0, stream);
    if (r != FA4CP_OK) return r;
    if (timed) FA4CP_CHECK_CUDA(cudaEventRecord(rc->tev[2 * rc->t_used++ + 1], st));
    if (s + 2 < S) FA4CP_CHECK_CUDA(cudaEventRecord(rc->ev_step[s], st));
  }
  return FA4CP_OK;
}
