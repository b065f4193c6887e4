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
// Two transports move the K/V:
//   * copy engine (preferred): each rank pushes the K/V it attended at step s-1 straight
//     into its right neighbour's receive slot with cudaMemcpyAsync over NVLink (a CUDA IPC
//     mapping of the neighbour's receive area), so the rotation takes no SM from the
//     attention kernel.  Arrival and slot release are 32-bit hop counters in the receive
//     areas, written into the peer's memory with cuStreamWriteValue32 (which fences the
//     stream's earlier writes first) and waited on locally with cuStreamWaitValue32.  The
//     order of operations is a plan (build_ce_plan) that a CPU test runs against a
//     multi-rank simulator for deadlocks and slot hazards;
//   * NCCL: send/recv on the executor's own communicator (ncclCommInitRank over the cp
//     group, NCCL rank = cp rank, unique id broadcast by the caller) into caller-provided
//     ping-pong buffers.  libnccl.so.2 is opened with dlopen, so the process's already
//     loaded NCCL (PyTorch's) is the one used.
#include <dlfcn.h>
#include <nccl.h>
#include <string.h>

#include <mutex>
#include <unordered_set>
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
constexpr int kDefaultSmReserve = 8;
// streams of the copy-engine plans: the caller's, the K and V copies, the slot releases, and
// a second K / V copy pair (direct pushes alternate destinations between the two pairs)
enum { ST_COMPUTE = 0, ST_COPY_K = 1, ST_COPY_V = 2, ST_RELEASE = 3, ST_COPY_K2 = 4,
       ST_COPY_V2 = 5, ST_COUNT = 6 };

struct RingComm {
  ncclComm_t comm = nullptr;
  int nranks = 0, rank = 0, device = 0;
  cudaStream_t stream = nullptr;       // high-priority comm stream
  cudaEvent_t ev_start = nullptr;      // the caller's stream reached the call
  cudaEvent_t ev_hop[kMaxRing] = {};   // hop s landed
  cudaEvent_t ev_step[kMaxRing] = {};  // attention of step s done (its K/V slot is free)
  int sm_reserve = kDefaultSmReserve;  // SMs the persistent attention grid leaves to NCCL
  // ring kernel: 0 never, 1 for f16 / bf16 (D 64, 128), 2 also for e4m3 (default), 3 also at
  // head_dim 256 (f16 / bf16, and bf16 q x e4m3 K/V)
  int fused = 2;
  // optional timing: 2 timing events per attention launch and per hop, filled in call order
  std::vector<cudaEvent_t> tev, hev;
  int t_used = 0, h_used = 0;
  // copy-engine transport
  bool ce = false;                       // transport: copy engine (else NCCL)
  bool direct = true;                    // direct pushes (else chained hops); set before alloc
  uint8_t* area = nullptr;               // own receive area (cudaMalloc)
  uint8_t* right = nullptr;              // right neighbour's area (IPC mapping)
  uint8_t* left = nullptr;               // left neighbour's area (== right when nranks == 2)
  uint8_t* peer[kMaxRing] = {};          // peer[d]: the area of rank rank + d (direct pushes)
  int64_t kv_cap = 0;                    // bytes of one K (or V) part of a slot
  int64_t nslots = 0;                    // slots per part in the area
  uint64_t hops = 0;                     // hops issued since the area was (re)allocated
  uint64_t calls = 0;                    // direct-push calls since the area was (re)allocated
  cudaStream_t cstream[ST_COUNT] = {};   // copy and release streams ([0]: the caller's)
  std::vector<cudaEvent_t> cev;          // plan events
};

// live ring handles: every entry point checks its handle here, so a destroyed, foreign or
// garbage handle is an argument error instead of a dereference
std::mutex g_rings_mu;
std::unordered_set<const RingComm*>& live_rings() {
  static std::unordered_set<const RingComm*> rings;
  return rings;
}
void register_ring(const RingComm* rc) {
  std::lock_guard<std::mutex> lock(g_rings_mu);
  live_rings().insert(rc);
}
bool unregister_ring(const RingComm* rc) {
  std::lock_guard<std::mutex> lock(g_rings_mu);
  return live_rings().erase(rc) > 0;
}
RingComm* ring_of(int64_t handle) {
  std::lock_guard<std::mutex> lock(g_rings_mu);
  RingComm* rc = reinterpret_cast<RingComm*>(handle);
  return live_rings().count(rc) ? rc : nullptr;
}

// restores the calling thread's SM reserve when a ring call returns
struct SmReserveScope {
  explicit SmReserveScope(int n) { set_sm_reserve(n); }
  ~SmReserveScope() { set_sm_reserve(0); }
};

void destroy_timing(RingComm* rc) {
  for (cudaEvent_t e : rc->tev)
    if (e) cudaEventDestroy(e);
  for (cudaEvent_t e : rc->hev)
    if (e) cudaEventDestroy(e);
  rc->tev.clear();
  rc->hev.clear();
  rc->t_used = rc->h_used = 0;
}

void close_peers(RingComm* rc) {
  std::unordered_set<uint8_t*> mapped;  // every mapping once (left == right when nranks == 2)
  for (int d = 1; d < kMaxRing; ++d)
    if (rc->peer[d]) mapped.insert(rc->peer[d]);
  if (rc->right) mapped.insert(rc->right);
  if (rc->left) mapped.insert(rc->left);
  for (uint8_t* m : mapped) cudaIpcCloseMemHandle(m);
  for (int d = 0; d < kMaxRing; ++d) rc->peer[d] = nullptr;
  rc->right = rc->left = nullptr;
  rc->ce = false;
}

void destroy_ring(RingComm* rc) {
  destroy_timing(rc);
  if (rc->area || rc->right) cudaDeviceSynchronize();
  close_peers(rc);
  if (rc->area) cudaFree(rc->area);
  for (int i = 1; i < ST_COUNT; ++i)
    if (rc->cstream[i]) cudaStreamDestroy(rc->cstream[i]);
  for (cudaEvent_t e : rc->cev)
    if (e) cudaEventDestroy(e);
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

// ---------------------------------------------------------------------------------------
// copy-engine transport: the plan
//
// Hop g (a counter over all hops of all calls since the area was allocated, from 1) carries
// one K/V shard; a call's hops g0+1 .. g0+S-1 land in the receiver's slots 0 .. S-2 (one
// slot per hop, so nothing is reused inside a call).  One call issues, in this host order:
//   RECORD start on the compute stream;
//   push(1) .. push(S-1), where push(s) (K on copy stream 1, V on copy stream 2) waits for
//     its data (the caller's stream for s = 1, else own ARRIVED >= g0+s-1), waits until the
//     right neighbour released its slot s-1 from the previous call (own FREED >= g0+s-(S-1),
//     once a previous call exists), copies into that slot, then writes the right neighbour's
//     ARRIVED = g0+s;
//   the attention: per-step launches (step s > 0 after own ARRIVED >= g0+s on the compute
//     stream) or one persistent ring kernel that waits for ARRIVED >= g0+s itself before it
//     reads slot s-1;
//   RECORD done; the release stream waits for the attention and the last push (which read
//     the own slots), then writes the left neighbour's FREED = g0+S-1;
//   the compute stream joins the copy and release streams.
// The pushes depend only on the previous call's releases and on earlier hops, never on
// this call's attention, so the whole rotation runs ahead of the compute, and no wait can
// close a cycle even if every stream of a rank ran in host order on one hardware queue.
// ---------------------------------------------------------------------------------------
enum { FLAG_ARRIVED = 0, FLAG_FREED = 1 };
enum { PEER_RIGHT = 0, PEER_LEFT = 1 };
constexpr int EV_START = 0;
constexpr int EV_DONE = 1;
constexpr int ev_vdone(int s) { return 2 + s; }
constexpr int ev_push(int s) { return 2 + kMaxRing + s; }
constexpr int EV_COPY_END = 2 + 2 * kMaxRing;
constexpr int EV_REL_END = 3 + 2 * kMaxRing;
constexpr int EV_COPY_END2 = 4 + 2 * kMaxRing;
constexpr int EV_COUNT = 5 + 2 * kMaxRing;
constexpr int64_t kSlotBase = 4096;           // receive slots start here in the area
// flags (32-bit words of the area's first 4 KiB): chained hops use ARRIVED at byte 0 and FREED
// at byte 128 (own 128-byte lines); direct pushes one arrival flag per slot (two sets of at
// most kMaxRing - 1 slots) from byte 256 and FREED[d] from byte 1024
constexpr int FLAG_SLOT0 = 2;
constexpr int FLAG_PEER_FREED0 = 2 + 2 * kMaxRing;
int64_t flag_offset(int64_t id) {
  if (id == FLAG_ARRIVED) return 0;
  if (id == FLAG_FREED) return 128;
  if (id < FLAG_PEER_FREED0) return 256 + 4 * (id - FLAG_SLOT0);
  return 1024 + 4 * (id - FLAG_PEER_FREED0);
}
static_assert(256 + 4 * 2 * kMaxRing <= 1024 && 1024 + 4 * kMaxRing <= kSlotBase, "flag layout");

using RingOp = fa4cp_ring_op;

void build_ce_plan(int S, int rank, uint64_t g0, bool fused, std::vector<RingOp>& ops) {
  (void)rank;  // the plan is the same on every rank; peers are implied (left / right)
  ops.clear();
  auto op = [&](int st, int kind, int64_t a = 0, int64_t b = 0, int64_t c = 0) {
    ops.push_back(RingOp{st, kind, a, b, c});
  };
  auto G = [&](int s) { return int64_t(uint32_t(g0 + uint64_t(s))); };  // counter value
  auto push = [&](int s) {
    for (int st : {ST_COPY_K, ST_COPY_V}) {
      if (s == 1)
        op(st, FA4CP_RING_OP_WAIT_EVENT, EV_START);
      else
        op(st, FA4CP_RING_OP_WAIT_FLAG, FLAG_ARRIVED, G(s - 1));
      if (g0 > 0)  // slot s-1 was last filled by the previous call's hop g0+s-(S-1)
        op(st, FA4CP_RING_OP_WAIT_FLAG, FLAG_FREED, int64_t(uint32_t(G(s) - (S - 1))));
      op(st, FA4CP_RING_OP_COPY, st == ST_COPY_K ? 0 : 1, s == 1 ? -1 : s - 2, s - 1);
    }
    op(ST_COPY_V, FA4CP_RING_OP_RECORD, ev_vdone(s));
    op(ST_COPY_K, FA4CP_RING_OP_WAIT_EVENT, ev_vdone(s));
    op(ST_COPY_K, FA4CP_RING_OP_WRITE_FLAG, PEER_RIGHT, FLAG_ARRIVED, G(s));
    op(ST_COPY_K, FA4CP_RING_OP_RECORD, ev_push(s));
  };
  if (S == 1) {
    op(ST_COMPUTE, FA4CP_RING_OP_ATTN, 0, -1);
    return;
  }
  op(ST_COMPUTE, FA4CP_RING_OP_RECORD, EV_START);
  for (int s = 1; s < S; ++s) push(s);
  if (fused) {
    op(ST_COMPUTE, FA4CP_RING_OP_ATTN_FUSED, S, G(0));
  } else {
    for (int s = 0; s < S; ++s) {
      if (s > 0) op(ST_COMPUTE, FA4CP_RING_OP_WAIT_FLAG, FLAG_ARRIVED, G(s));
      op(ST_COMPUTE, FA4CP_RING_OP_ATTN, s, s == 0 ? -1 : s - 1);
    }
  }
  op(ST_COMPUTE, FA4CP_RING_OP_RECORD, EV_DONE);
  op(ST_RELEASE, FA4CP_RING_OP_WAIT_EVENT, EV_DONE);
  op(ST_RELEASE, FA4CP_RING_OP_WAIT_EVENT, ev_push(S - 1));
  op(ST_RELEASE, FA4CP_RING_OP_WRITE_FLAG, PEER_LEFT, FLAG_FREED, G(S - 1));
  op(ST_COPY_K, FA4CP_RING_OP_RECORD, EV_COPY_END);
  op(ST_RELEASE, FA4CP_RING_OP_RECORD, EV_REL_END);
  op(ST_COMPUTE, FA4CP_RING_OP_WAIT_EVENT, EV_COPY_END);
  op(ST_COMPUTE, FA4CP_RING_OP_WAIT_EVENT, EV_REL_END);
}

// ---------------------------------------------------------------------------------------
// copy-engine transport, direct pushes: the plan of call number n (>= 1)
//
// Over NVSwitch every GPU reaches every peer at full bandwidth, so instead of forwarding
// shards hop by hop (step s then waits for s - 1 transfers in a row), each rank pushes its
// own K/V straight to every other rank at the start of the call:
//   RECORD start on the compute stream;
//   for d = 1 .. S-1 (rank + d attends this rank's K/V at its step d), on copy pair (d-1) % 2:
//     both streams wait for start and, from call 3 on, for FREED[d] >= n - 2 (rank + d is done
//     with the same slot set, used by call n - 2); K and V go to slot set*(S-1) + d-1 of
//     rank + d (set = n % 2); then rank + d's arrival flag of that slot := n;
//   the attention: per-step launches (step s > 0 after its slot's flag >= n on the compute
//     stream) or the ring kernel, which waits for each slot's flag itself;
//   RECORD done; the release stream waits for it and sets FREED[s] := n at rank - s for
//     every s (the source of the slot this rank read at step s);
//   the compute stream joins the copy streams (they read the caller's K/V); the releases run
//     on in the background.
// A push depends only on the call's start and on releases two calls back, and an attention
// only on this call's pushes, so no wait can close a cycle even if every stream of every rank
// ran in host order on one queue.
// ---------------------------------------------------------------------------------------
void build_ce_direct_plan(int S, int rank, uint64_t n, bool fused, std::vector<RingOp>& ops) {
  (void)rank;
  ops.clear();
  auto op = [&](int st, int kind, int64_t a = 0, int64_t b = 0, int64_t c = 0) {
    ops.push_back(RingOp{st, kind, a, b, c});
  };
  const int64_t N = int64_t(uint32_t(n));  // flag value of this call
  if (S == 1) {
    op(ST_COMPUTE, FA4CP_RING_OP_ATTN, 0, -1);
    return;
  }
  const int64_t set0 = int64_t(n & 1) * (S - 1);  // first slot of this call's set
  op(ST_COMPUTE, FA4CP_RING_OP_RECORD, EV_START);
  for (int d = 1; d < S; ++d) {
    const int kst = (d - 1) % 2 ? ST_COPY_K2 : ST_COPY_K;
    const int vst = (d - 1) % 2 ? ST_COPY_V2 : ST_COPY_V;
    const int64_t slot = set0 + d - 1;
    for (int st : {kst, vst}) {
      op(st, FA4CP_RING_OP_WAIT_EVENT, EV_START);
      if (n > 2) op(st, FA4CP_RING_OP_WAIT_FLAG, FLAG_PEER_FREED0 + d, int64_t(uint32_t(n - 2)));
      op(st, FA4CP_RING_OP_COPY_TO, st == kst ? 0 : 1, d, slot);
    }
    op(vst, FA4CP_RING_OP_RECORD, ev_vdone(d));
    op(kst, FA4CP_RING_OP_WAIT_EVENT, ev_vdone(d));
    op(kst, FA4CP_RING_OP_WRITE_PEER, d, FLAG_SLOT0 + slot, N);
    op(kst, FA4CP_RING_OP_RECORD, ev_push(d));
  }
  if (fused) {
    op(ST_COMPUTE, FA4CP_RING_OP_ATTN_FUSED_SLOTS, S, N, set0);
  } else {
    for (int s = 0; s < S; ++s) {
      if (s > 0) op(ST_COMPUTE, FA4CP_RING_OP_WAIT_FLAG, FLAG_SLOT0 + set0 + s - 1, N);
      op(ST_COMPUTE, FA4CP_RING_OP_ATTN, s, s == 0 ? -1 : set0 + s - 1);
    }
  }
  op(ST_COMPUTE, FA4CP_RING_OP_RECORD, EV_DONE);
  op(ST_RELEASE, FA4CP_RING_OP_WAIT_EVENT, EV_DONE);
  for (int s = 1; s < S; ++s)
    op(ST_RELEASE, FA4CP_RING_OP_WRITE_PEER, S - s, FLAG_PEER_FREED0 + s, N);
  // the caller's stream joins the copy streams, which read its K/V; the releases only write
  // flags in the peers' memory and run on in the background (the next call's release follows
  // them on the same stream, and a push waits for its destination's release itself)
  op(ST_COPY_K, FA4CP_RING_OP_RECORD, EV_COPY_END);
  if (S > 2) op(ST_COPY_K2, FA4CP_RING_OP_RECORD, EV_COPY_END2);
  op(ST_COMPUTE, FA4CP_RING_OP_WAIT_EVENT, EV_COPY_END);
  if (S > 2) op(ST_COMPUTE, FA4CP_RING_OP_WAIT_EVENT, EV_COPY_END2);
}

using StreamWaitValue32Fn = CUresult (*)(CUstream, CUdeviceptr, cuuint32_t, unsigned int);
using StreamWriteValue32Fn = CUresult (*)(CUstream, CUdeviceptr, cuuint32_t, unsigned int);

struct StreamMemOps {
  StreamWaitValue32Fn wait = nullptr;
  StreamWriteValue32Fn write = nullptr;
};

StreamMemOps* stream_mem_ops() {
  static StreamMemOps ops;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuStreamWaitValue32", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      ops.wait = reinterpret_cast<StreamWaitValue32Fn>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuStreamWriteValue32", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      ops.write = reinterpret_cast<StreamWriteValue32Fn>(p);
  });
  return (ops.wait && ops.write) ? &ops : nullptr;
}

}  // namespace
}  // namespace fa4cp

using namespace fa4cp;

extern "C" int fa4cp_ring_ce_plan(int32_t nranks, int32_t rank, int64_t g0, int32_t fused,
                                  fa4cp_ring_op* ops, int32_t capacity) {
  FA4CP_CHECK_ARG(g0 >= 0, "negative hop count");
  FA4CP_CHECK_ARG(nranks >= 1 && nranks <= kMaxRing && rank >= 0 && rank < nranks,
                  "bad ring size %d / rank %d", nranks, rank);
  std::vector<RingOp> plan;
  build_ce_plan(nranks, rank, uint64_t(g0), fused != 0, plan);
  FA4CP_CHECK_ARG(ops == nullptr || capacity >= int32_t(plan.size()),
                  "capacity %d < %d plan entries", capacity, int(plan.size()));
  if (ops != nullptr) memcpy(ops, plan.data(), plan.size() * sizeof(RingOp));
  return int32_t(plan.size());
}

extern "C" int fa4cp_ring_ce_direct_plan(int32_t nranks, int32_t rank, int64_t call,
                                         int32_t fused, fa4cp_ring_op* ops, int32_t capacity) {
  FA4CP_CHECK_ARG(call >= 1, "call numbers start at 1");
  FA4CP_CHECK_ARG(nranks >= 1 && nranks <= kMaxRing && rank >= 0 && rank < nranks,
                  "bad ring size %d / rank %d", nranks, rank);
  std::vector<RingOp> plan;
  build_ce_direct_plan(nranks, rank, uint64_t(call), fused != 0, plan);
  FA4CP_CHECK_ARG(ops == nullptr || capacity >= int32_t(plan.size()),
                  "capacity %d < %d plan entries", capacity, int(plan.size()));
  if (ops != nullptr) memcpy(ops, plan.data(), plan.size() * sizeof(RingOp));
  return int32_t(plan.size());
}

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
  FA4CP_CHECK_ARG(handle_out != nullptr, "null argument");
  FA4CP_CHECK_ARG(nranks >= 1 && nranks <= kMaxRing && rank >= 0 && rank < nranks,
                  "bad ring size %d / rank %d (at most %d ranks)", nranks, rank, kMaxRing);
  NcclApi* api = nccl_api();
  FA4CP_CHECK_ARG(id == nullptr || api != nullptr, "libnccl.so.2 could not be loaded");
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
  for (int i = 1; ce == cudaSuccess && i < ST_COUNT; ++i)
    ce = cudaStreamCreateWithPriority(&rc->cstream[i], cudaStreamNonBlocking, hi);
  rc->cev.assign(EV_COUNT, nullptr);
  for (int i = 0; ce == cudaSuccess && i < EV_COUNT; ++i)
    ce = cudaEventCreateWithFlags(&rc->cev[i], cudaEventDisableTiming);
  if (ce != cudaSuccess) {
    set_last_error("ring stream/event creation failed: %s", cudaGetErrorString(ce));
    destroy_ring(rc);
    return FA4CP_ERR_CUDA;
  }
  if (nranks > 1 && id != nullptr) {
    ncclUniqueId uid;
    memcpy(&uid, id, sizeof(uid));
    ncclResult_t r = api->CommInitRank(&rc->comm, nranks, uid, rank);
    if (r != ncclSuccess) {
      rc->comm = nullptr;
      destroy_ring(rc);
      return nccl_fail(api, "ncclCommInitRank", r);
    }
  }
  register_ring(rc);
  *handle_out = reinterpret_cast<int64_t>(rc);
  return FA4CP_OK;
}

extern "C" int fa4cp_ring_comm_destroy(int64_t handle) {
  FA4CP_CHECK_ARG(handle != 0, "null ring handle");
  RingComm* rc = ring_of(handle);
  FA4CP_CHECK_ARG(rc != nullptr && unregister_ring(rc), "unknown ring handle");
  NcclApi* api = nccl_api();
  cudaStreamSynchronize(rc->stream);
  if (api != nullptr && rc->comm != nullptr) api->CommDestroy(rc->comm);
  destroy_ring(rc);
  return FA4CP_OK;
}

extern "C" int fa4cp_ring_ipc_alloc(int64_t handle, int64_t kv_capacity, uint8_t* ipc_out) {
  FA4CP_CHECK_ARG(handle != 0 && ipc_out != nullptr, "null argument");
  FA4CP_CHECK_ARG(kv_capacity > 0 && kv_capacity <= (int64_t(1) << 40), "bad kv_capacity");
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "CUDA IPC handles are 64 bytes");
  RingComm* rc = ring_of(handle);
  FA4CP_CHECK_ARG(rc != nullptr, "unknown ring handle");
  FA4CP_CHECK_CUDA(cudaDeviceSynchronize());
  close_peers(rc);
  if (rc->area) {
    FA4CP_CHECK_CUDA(cudaFree(rc->area));
    rc->area = nullptr;
  }
  const int64_t cap = (kv_capacity + 255) / 256 * 256;
  void* p = nullptr;
  // per part (K, V): one slot per hop, times two alternating sets for direct pushes
  const int64_t nslots = (rc->nranks > 1 ? rc->nranks - 1 : 1) * (rc->direct ? 2 : 1);
  FA4CP_CHECK_CUDA(cudaMalloc(&p, size_t(kSlotBase + 2 * nslots * cap)));
  rc->area = static_cast<uint8_t*>(p);
  rc->kv_cap = cap;
  rc->nslots = nslots;
  rc->hops = 0;
  rc->calls = 0;
  FA4CP_CHECK_CUDA(cudaMemset(rc->area, 0, size_t(kSlotBase)));
  FA4CP_CHECK_CUDA(cudaDeviceSynchronize());
  cudaIpcMemHandle_t h;
  FA4CP_CHECK_CUDA(cudaIpcGetMemHandle(&h, rc->area));
  memcpy(ipc_out, &h, sizeof(h));
  return FA4CP_OK;
}

extern "C" int fa4cp_ring_ipc_open(int64_t handle, const uint8_t* left_ipc,
                                   const uint8_t* right_ipc) {
  FA4CP_CHECK_ARG(handle != 0 && left_ipc != nullptr && right_ipc != nullptr, "null argument");
  RingComm* rc = ring_of(handle);
  FA4CP_CHECK_ARG(rc != nullptr, "unknown ring handle");
  FA4CP_CHECK_ARG(rc->nranks > 1, "a ring of one rank has no neighbours");
  FA4CP_CHECK_ARG(rc->area != nullptr, "fa4cp_ring_ipc_alloc must come first");
  FA4CP_CHECK_ARG(stream_mem_ops() != nullptr,
                  "cuStreamWaitValue32/cuStreamWriteValue32 are not available");
  close_peers(rc);
  cudaIpcMemHandle_t hr, hl;
  memcpy(&hr, right_ipc, sizeof(hr));
  memcpy(&hl, left_ipc, sizeof(hl));
  void* pr = nullptr;
  FA4CP_CHECK_CUDA(cudaIpcOpenMemHandle(&pr, hr, cudaIpcMemLazyEnablePeerAccess));
  rc->right = static_cast<uint8_t*>(pr);
  if (memcmp(&hr, &hl, sizeof(hr)) == 0) {
    rc->left = rc->right;
  } else {
    void* pl = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&pl, hl, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      close_peers(rc);
      set_last_error("cudaIpcOpenMemHandle(left) failed: %s", cudaGetErrorString(e));
      return FA4CP_ERR_CUDA;
    }
    rc->left = static_cast<uint8_t*>(pl);
  }
  rc->peer[1] = rc->right;
  rc->peer[rc->nranks - 1] = rc->left;
  rc->ce = true;
  return FA4CP_OK;
}

extern "C" int fa4cp_ring_ipc_open_all(int64_t handle, const uint8_t* ipc_handles) {
  FA4CP_CHECK_ARG(handle != 0 && ipc_handles != nullptr, "null argument");
  RingComm* rc = ring_of(handle);
  FA4CP_CHECK_ARG(rc != nullptr, "unknown ring handle");
  FA4CP_CHECK_ARG(rc->nranks > 1, "a ring of one rank has no peers");
  FA4CP_CHECK_ARG(rc->area != nullptr, "fa4cp_ring_ipc_alloc must come first");
  FA4CP_CHECK_ARG(stream_mem_ops() != nullptr,
                  "cuStreamWaitValue32/cuStreamWriteValue32 are not available");
  close_peers(rc);
  for (int d = 1; d < rc->nranks; ++d) {
    cudaIpcMemHandle_t h;
    memcpy(&h, ipc_handles + 64 * ((rc->rank + d) % rc->nranks), sizeof(h));
    void* ptr = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      close_peers(rc);
      set_last_error("cudaIpcOpenMemHandle(rank %d) failed: %s", (rc->rank + d) % rc->nranks,
                     cudaGetErrorString(e));
      return FA4CP_ERR_CUDA;
    }
    rc->peer[d] = static_cast<uint8_t*>(ptr);
  }
  rc->right = rc->peer[1];
  rc->left = rc->peer[rc->nranks - 1];
  rc->ce = true;
  return FA4CP_OK;
}

extern "C" int fa4cp_ring_set_direct(int64_t handle, int32_t on) {
  FA4CP_CHECK_ARG(handle != 0, "null ring handle");
  FA4CP_CHECK_ARG(on == 0 || on == 1, "direct must be 0 or 1");
  RingComm* rc = ring_of(handle);
  FA4CP_CHECK_ARG(rc != nullptr, "unknown ring handle");
  FA4CP_CHECK_ARG(rc->area == nullptr, "set the push mode before fa4cp_ring_ipc_alloc");
  rc->direct = on != 0;
  return FA4CP_OK;
}

extern "C" int fa4cp_ring_ipc_close(int64_t handle) {
  FA4CP_CHECK_ARG(handle != 0, "null ring handle");
  RingComm* rc = ring_of(handle);
  FA4CP_CHECK_ARG(rc != nullptr, "unknown ring handle");
  FA4CP_CHECK_CUDA(cudaDeviceSynchronize());
  close_peers(rc);
  return FA4CP_OK;
}

extern "C" int fa4cp_ring_timing(int64_t handle, int32_t max_launches) {
  FA4CP_CHECK_ARG(handle != 0, "null ring handle");
  FA4CP_CHECK_ARG(max_launches >= 0 && max_launches <= (1 << 16), "bad max_launches %d",
                  max_launches);
  RingComm* rc = ring_of(handle);
  FA4CP_CHECK_ARG(rc != nullptr, "unknown ring handle");
  destroy_timing(rc);
  rc->tev.assign(2 * size_t(max_launches), nullptr);
  rc->hev.assign(2 * size_t(max_launches), nullptr);
  for (auto* vec : {&rc->tev, &rc->hev}) {
    for (auto& e : *vec) {
      cudaError_t ce = cudaEventCreate(&e);
      if (ce != cudaSuccess) {
        set_last_error("cudaEventCreate failed: %s", cudaGetErrorString(ce));
        destroy_timing(rc);
        return FA4CP_ERR_CUDA;
      }
    }
  }
  return FA4CP_OK;
}

extern "C" int fa4cp_ring_set_fused(int64_t handle, int32_t fused) {
  FA4CP_CHECK_ARG(handle != 0, "null ring handle");
  FA4CP_CHECK_ARG(fused >= 0 && fused <= 3, "fused mode %d not in 0..3", fused);
  RingComm* rc = ring_of(handle);
  FA4CP_CHECK_ARG(rc != nullptr, "unknown ring handle");
  rc->fused = fused;
  return FA4CP_OK;
}

extern "C" int fa4cp_ring_set_sm_reserve(int64_t handle, int32_t sm_reserve) {
  FA4CP_CHECK_ARG(handle != 0, "null ring handle");
  FA4CP_CHECK_ARG(sm_reserve >= 0 && sm_reserve <= 64, "sm_reserve %d out of [0, 64]", sm_reserve);
  RingComm* rc = ring_of(handle);
  FA4CP_CHECK_ARG(rc != nullptr, "unknown ring handle");
  rc->sm_reserve = sm_reserve;
  return FA4CP_OK;
}

extern "C" int fa4cp_ring_timeline(int64_t handle, float* attn_ms, int32_t max_attn,
                                   float* hop_ms, int32_t max_hops, int32_t* n_attn,
                                   int32_t* n_hops) {
  FA4CP_CHECK_ARG(handle != 0 && n_attn != nullptr && n_hops != nullptr, "null argument");
  RingComm* rc = ring_of(handle);
  FA4CP_CHECK_ARG(rc != nullptr, "unknown ring handle");
  *n_attn = *n_hops = 0;
  if (rc->t_used == 0) return FA4CP_OK;
  cudaEvent_t t0 = rc->tev[0];
  auto rel = [&](cudaEvent_t e, float* dst) -> int {
    FA4CP_CHECK_CUDA(cudaEventSynchronize(e));
    FA4CP_CHECK_CUDA(cudaEventElapsedTime(dst, t0, e));
    return FA4CP_OK;
  };
  int r;
  const int na = rc->t_used < max_attn ? rc->t_used : max_attn;
  for (int i = 0; i < na && attn_ms != nullptr; ++i)
    if ((r = rel(rc->tev[2 * i], attn_ms + 2 * i)) || (r = rel(rc->tev[2 * i + 1], attn_ms + 2 * i + 1)))
      return r;
  const int nh = rc->h_used < max_hops ? rc->h_used : max_hops;
  for (int i = 0; i < nh && hop_ms != nullptr; ++i)
    if ((r = rel(rc->hev[2 * i], hop_ms + 2 * i)) || (r = rel(rc->hev[2 * i + 1], hop_ms + 2 * i + 1)))
      return r;
  *n_attn = attn_ms != nullptr ? na : 0;
  *n_hops = hop_ms != nullptr ? nh : 0;
  return FA4CP_OK;
}

extern "C" int fa4cp_ring_timing_read(int64_t handle, double* total_ms, int32_t* launches) {
  FA4CP_CHECK_ARG(handle != 0 && total_ms != nullptr && launches != nullptr, "null argument");
  RingComm* rc = ring_of(handle);
  FA4CP_CHECK_ARG(rc != nullptr, "unknown ring handle");
  double sum = 0.0;
  for (int i = 0; i < rc->t_used; ++i) {
    FA4CP_CHECK_CUDA(cudaEventSynchronize(rc->tev[2 * i + 1]));
    float ms = 0.f;
    FA4CP_CHECK_CUDA(cudaEventElapsedTime(&ms, rc->tev[2 * i], rc->tev[2 * i + 1]));
    sum += ms;
  }
  *total_ms = sum;
  *launches = rc->t_used;
  rc->t_used = rc->h_used = 0;
  return FA4CP_OK;
}

namespace {

// Issues the copy-engine plan of one call (build_ce_plan, or build_ce_direct_plan for direct
// pushes) on the caller's stream `st` and the ring's copy / release streams.
template <class AttnStep, class AttnFused>
int run_ce(RingComm* rc, AttnStep& attn_step, AttnFused* attn_fused, const void* k,
           const void* v, int64_t kv_bytes, cudaStream_t st) {
  FA4CP_CHECK_ARG(kv_bytes <= rc->kv_cap, "K/V shard of %lld bytes exceeds the receive slots "
                  "(%lld bytes; reallocate with fa4cp_ring_ipc_alloc)",
                  static_cast<long long>(kv_bytes), static_cast<long long>(rc->kv_cap));
  StreamMemOps* mem = stream_mem_ops();
  FA4CP_CHECK_ARG(mem != nullptr, "stream memory operations are not available");
  const bool direct = rc->direct;
  FA4CP_CHECK_ARG(rc->nslots == (rc->nranks - 1) * (direct ? 2 : 1),
                  "the receive area was allocated for the other push mode");
  for (int d = 1; direct && d < rc->nranks; ++d)
    FA4CP_CHECK_ARG(rc->peer[d] != nullptr, "direct pushes need every peer mapped "
                    "(fa4cp_ring_ipc_open_all)");
  std::vector<RingOp> plan;
  const uint64_t call = rc->calls + 1;
  if (direct)
    build_ce_direct_plan(rc->nranks, rc->rank, call, attn_fused != nullptr, plan);
  else
    build_ce_plan(rc->nranks, rc->rank, rc->hops, attn_fused != nullptr, plan);
  cudaStream_t streams[ST_COUNT];
  streams[ST_COMPUTE] = st;
  for (int i = 1; i < ST_COUNT; ++i) streams[i] = rc->cstream[i];
  // K slots 0 .. nslots-1, then V slots
  auto slot = [&](uint8_t* area, int64_t idx, int64_t part) {
    return area + kSlotBase + (part * rc->nslots + idx) * rc->kv_cap;
  };
  auto flag = [&](uint8_t* area, int64_t id) {
    return reinterpret_cast<CUdeviceptr>(area + flag_offset(id));
  };
  for (const RingOp& o : plan) {
    cudaStream_t cs = streams[o.stream];
    switch (o.kind) {
      case FA4CP_RING_OP_RECORD: {
        FA4CP_CHECK_CUDA(cudaEventRecord(rc->cev[o.a], cs));
        const bool push_end = o.a >= ev_push(0) && o.a < ev_push(kMaxRing);
        if (push_end && rc->h_used < int(rc->hev.size() / 2))
          FA4CP_CHECK_CUDA(cudaEventRecord(rc->hev[2 * rc->h_used++ + 1], cs));
        break;
      }
      case FA4CP_RING_OP_WAIT_EVENT:
        FA4CP_CHECK_CUDA(cudaStreamWaitEvent(cs, rc->cev[o.a], 0));
        break;
      case FA4CP_RING_OP_WAIT_FLAG: {
        CUresult e = mem->wait(cs, flag(rc->area, o.a), cuuint32_t(o.b), CU_STREAM_WAIT_VALUE_GEQ);
        FA4CP_CHECK_ARG(e == CUDA_SUCCESS, "cuStreamWaitValue32 failed (CUresult %d)", int(e));
        break;
      }
      case FA4CP_RING_OP_WRITE_FLAG: {
        uint8_t* peer = o.a == PEER_RIGHT ? rc->right : rc->left;
        CUresult e = mem->write(cs, flag(peer, o.b), cuuint32_t(o.c), CU_STREAM_WRITE_VALUE_DEFAULT);
        FA4CP_CHECK_ARG(e == CUDA_SUCCESS, "cuStreamWriteValue32 failed (CUresult %d)", int(e));
        break;
      }
      case FA4CP_RING_OP_WRITE_PEER: {
        CUresult e = mem->write(cs, flag(rc->peer[o.a], o.b), cuuint32_t(o.c),
                                CU_STREAM_WRITE_VALUE_DEFAULT);
        FA4CP_CHECK_ARG(e == CUDA_SUCCESS, "cuStreamWriteValue32 failed (CUresult %d)", int(e));
        break;
      }
      case FA4CP_RING_OP_COPY: {
        const void* src = o.b < 0 ? (o.a == 0 ? k : v) : slot(rc->area, o.b, o.a);
        if (o.a == 0 && rc->h_used < int(rc->hev.size() / 2))
          FA4CP_CHECK_CUDA(cudaEventRecord(rc->hev[2 * rc->h_used], cs));
        FA4CP_CHECK_CUDA(cudaMemcpyAsync(slot(rc->right, o.c, o.a), src, size_t(kv_bytes),
                                         cudaMemcpyDeviceToDevice, cs));
        break;
      }
      case FA4CP_RING_OP_COPY_TO: {
        if (o.a == 0 && rc->h_used < int(rc->hev.size() / 2))
          FA4CP_CHECK_CUDA(cudaEventRecord(rc->hev[2 * rc->h_used], cs));
        FA4CP_CHECK_CUDA(cudaMemcpyAsync(slot(rc->peer[o.b], o.c, o.a), o.a == 0 ? k : v,
                                         size_t(kv_bytes), cudaMemcpyDeviceToDevice, cs));
        break;
      }
      case FA4CP_RING_OP_ATTN: {
        const void* kk = o.b < 0 ? k : slot(rc->area, o.b, 0);
        const void* vv = o.b < 0 ? v : slot(rc->area, o.b, 1);
        int r = attn_step(int(o.a), kk, vv);
        if (r != FA4CP_OK) return r;
        break;
      }
      case FA4CP_RING_OP_ATTN_FUSED: {
        int r = (*attn_fused)(slot(rc->area, 0, 0), slot(rc->area, 0, 1), rc->kv_cap,
                              reinterpret_cast<const uint32_t*>(rc->area + flag_offset(FLAG_ARRIVED)),
                              uint32_t(o.b), 0, 1);
        if (r != FA4CP_OK) return r;
        break;
      }
      case FA4CP_RING_OP_ATTN_FUSED_SLOTS: {
        int r = (*attn_fused)(slot(rc->area, o.c, 0), slot(rc->area, o.c, 1), rc->kv_cap,
                              reinterpret_cast<const uint32_t*>(rc->area + flag_offset(FLAG_SLOT0 + o.c)),
                              uint32_t(o.b), 1, 0);
        if (r != FA4CP_OK) return r;
        break;
      }
      default:
        set_last_error("unknown ring plan operation %d", o.kind);
        return FA4CP_ERR_INVALID;
    }
  }
  if (direct)
    rc->calls = call;
  else
    rc->hops += uint64_t(rc->nranks - 1);
  return FA4CP_OK;
}

}  // namespace

extern "C" int fa4cp_ring_attn_fwd(int64_t handle, const void* q, const void* k, const void* v,
                                   void* kv_bufs, int64_t kv_bufs_bytes, void* out, float* lse,
                                   const int32_t* cu, int32_t nseq, int32_t max_seqlen,
                                   int64_t total, int32_t num_heads_q, int32_t num_heads_kv,
                                   int32_t head_dim, int32_t q_dtype, int32_t kv_dtype,
                                   float softmax_scale, const float* q_descale,
                                   const float* k_descales, const float* v_descales,
                                   void* workspace, int64_t workspace_bytes, void* stream) {
  FA4CP_CHECK_ARG(handle != 0, "null ring handle");
  RingComm* rc = ring_of(handle);
  FA4CP_CHECK_ARG(rc != nullptr, "unknown ring handle");
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
  int dev = 0;
  FA4CP_CHECK_CUDA(cudaGetDevice(&dev));
  FA4CP_CHECK_ARG(dev == rc->device, "current device %d is not the ring's device %d", dev,
                  rc->device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  // attention of step s on the given K/V, merged into (out, lse) for s > 0
  auto attn_step = [&](int s, const void* kk, const void* vv) -> int {
    const int src = (rank - s + S) % S;
    const int pattern = s == 0 ? FA4CP_PATTERN_VARLEN
                               : (s > rank ? FA4CP_PATTERN_BACK_Q : FA4CP_PATTERN_FRONT_KV);
    const int q_rows = pattern == FA4CP_PATTERN_BACK_Q ? (max_seqlen + 1) / 2 : max_seqlen;
    const float* kd = k_descales ? k_descales + int64_t(src) * num_heads_kv : nullptr;
    const float* vd = v_descales ? v_descales + int64_t(src) * num_heads_kv : nullptr;
    const bool timed = rc->t_used < int(rc->tev.size() / 2);
    if (timed) FA4CP_CHECK_CUDA(cudaEventRecord(rc->tev[2 * rc->t_used], st));
    int r;
    if (mixed)
      r = fa4cp_attn_fwd_kv8(q, kk, vv, out, lse, cu, cu, nseq, q_rows, total, total, num_heads_q,
                             num_heads_kv, head_dim, q_dtype, pattern, s == 0, softmax_scale, kd,
                             vd, s > 0, workspace, workspace_bytes, stream);
    else
      r = fa4cp_attn_fwd(q, kk, vv, out, lse, cu, cu, nseq, q_rows, total, total, num_heads_q,
                         num_heads_kv, head_dim, q_dtype, out_dtype, pattern, s == 0,
                         softmax_scale, q_descale, kd, vd, s > 0, stream);
    if (r != FA4CP_OK) return r;
    if (timed) FA4CP_CHECK_CUDA(cudaEventRecord(rc->tev[2 * rc->t_used++ + 1], st));
    return FA4CP_OK;
  };

  // the persistent ring kernel: every step in one launch (f16 / bf16 D 64 or 128, e4m3 D 128)
  // With direct pushes, f16 / bf16 operands and S >= 8 the forward is two launches: step 0
  // (the local K/V, causal) on its own, then the ring kernel over the remote steps, merged into
  // it.  Step 0 is 1/S of the rank's work and needs no transfer, so the remote walk starts only
  // once the first pushes have landed: with one launch, the first wave of CTAs reaches the
  // remote steps after its own short step-0 tiles and waits for slots still in flight.  With
  // fewer ranks step 0 is a large share of the work and the second launch's tail and merge
  // cost more than they hide (cfg2 at cp=2: 2064 against 2240-2316 TF/s in one launch).
  // bf16 q x e4m3 K/V at head_dim 256 (the ring kernel fa4cp_ring_attn_fused_mixed): the rank
  // converts its K/V to bf16 once (exact: e4m3 values are bf16 values) into the workspace,
  // pushes those images and the kernel applies the per-source descales.  The pushes carry twice
  // the e4m3 bytes; at the shapes this serves (cfg5: 64 MB per rank against a forward of tens of
  // ms) they stay hidden behind step 0.
  const bool mixed_fused = mixed && rc->fused >= 3 && head_dim == 256;
  const void* k_loc = k;
  const void* v_loc = v;
  int64_t push_bytes = kv_bytes;
  const int32_t fused_dtype = mixed ? FA4CP_DTYPE_BF16 : q_dtype;
  auto attn_fused = [&](const void* sk, const void* sv, int64_t stride, const uint32_t* arrived,
                        uint32_t base, int32_t flag_stride, int32_t flag_step) -> int {
    const bool timed = rc->t_used < int(rc->tev.size() / 2);
    if (timed) FA4CP_CHECK_CUDA(cudaEventRecord(rc->tev[2 * rc->t_used], st));
    const bool two_pass = S >= 8 && flag_stride == 1 && q_dtype != FA4CP_DTYPE_E4M3 &&
                          head_dim != 256;
    int r = FA4CP_OK;
    if (two_pass)
      r = fa4cp_attn_fwd(q, k, v, out, lse, cu, cu, nseq, max_seqlen, total, total, num_heads_q,
                         num_heads_kv, head_dim, q_dtype, out_dtype, FA4CP_PATTERN_VARLEN, 1,
                         softmax_scale, nullptr, nullptr, nullptr, 0, stream);
    if (r == FA4CP_OK)
      r = ring_attn_fused_flags(q, k_loc, v_loc, sk, sv, stride, out, lse, cu, nseq, max_seqlen,
                                total, num_heads_q, num_heads_kv, head_dim, fused_dtype,
                                softmax_scale, q_descale, k_descales, v_descales, S, rank, arrived,
                                base, flag_stride, flag_step, two_pass ? 1 : 0, two_pass ? 1 : 0,
                                stream);
    if (r != FA4CP_OK) return r;
    if (timed) FA4CP_CHECK_CUDA(cudaEventRecord(rc->tev[2 * rc->t_used++ + 1], st));
    return FA4CP_OK;
  };
  const bool fusable =
      mixed_fused ||
      (q_dtype == kv_dtype &&
       ((rc->fused >= 1 && (q_dtype == FA4CP_DTYPE_BF16 || q_dtype == FA4CP_DTYPE_F16) &&
         (head_dim == 64 || head_dim == 128 || (head_dim == 256 && rc->fused >= 3))) ||
        (rc->fused >= 2 && q_dtype == FA4CP_DTYPE_E4M3 && head_dim == 128)));
  if (mixed_fused && (S == 1 || rc->ce)) {
    push_bytes = total * num_heads_kv * int64_t(head_dim) * 2;
    FA4CP_CHECK_ARG(workspace != nullptr && workspace_bytes >= 2 * push_bytes &&
                        uintptr_t(workspace) % 16 == 0,
                    "bf16 x e4m3 K/V: the workspace must hold the bf16 K and V (%lld bytes, "
                    "16-byte aligned)", static_cast<long long>(2 * push_bytes));
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    int r = launch_dequant_e4m3(k, nullptr, ws, total, num_heads_kv, head_dim, st);
    if (r == FA4CP_OK)
      r = launch_dequant_e4m3(v, nullptr, ws + push_bytes, total, num_heads_kv, head_dim, st);
    if (r != FA4CP_OK) return r;
    k_loc = ws;
    v_loc = ws + push_bytes;
  }
  if (S == 1)
    return fusable ? attn_fused(nullptr, nullptr, 0, nullptr, 0, 0, 1) : attn_step(0, k, v);
  if (rc->ce)
    return run_ce(rc, attn_step, fusable ? &attn_fused : nullptr, k_loc, v_loc, push_bytes, st);

  // ---- NCCL transport
  FA4CP_CHECK_ARG(kv_bufs != nullptr && kv_bufs_bytes >= 4 * kv_bytes,
                  "kv_bufs must hold two slots of K and V (%lld bytes)",
                  static_cast<long long>(4 * kv_bytes));
  FA4CP_CHECK_ARG(uintptr_t(kv_bufs) % 16 == 0, "kv_bufs must be 16-byte aligned");
  NcclApi* api = nccl_api();
  FA4CP_CHECK_ARG(api != nullptr && rc->comm != nullptr, "the ring has no NCCL communicator");
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
    const bool timed = rc->h_used < int(rc->hev.size() / 2);
    if (timed) FA4CP_CHECK_CUDA(cudaEventRecord(rc->hev[2 * rc->h_used], rc->stream));
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
    if (timed) FA4CP_CHECK_CUDA(cudaEventRecord(rc->hev[2 * rc->h_used++ + 1], rc->stream));
    return FA4CP_OK;
  };

  int r = FA4CP_OK;
  SmReserveScope reserve(rc->sm_reserve);
  if ((r = hop(1)) != FA4CP_OK) return r;  // hop 1 overlaps the local step
  for (int s = 0; s < S; ++s) {
    if (s > 0) {
      FA4CP_CHECK_CUDA(cudaStreamWaitEvent(st, rc->ev_hop[s], 0));
      if (s + 1 < S && (r = hop(s + 1)) != FA4CP_OK) return r;
    }
    if ((r = attn_step(s, step_k(s), step_v(s))) != FA4CP_OK) return r;
    if (s + 2 < S) FA4CP_CHECK_CUDA(cudaEventRecord(rc->ev_step[s], st));
  }
  return FA4CP_OK;
}
