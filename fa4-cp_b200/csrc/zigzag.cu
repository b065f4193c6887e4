// Zig-zag gather/scatter kernels and device-side half indices.
//
// Layout (fa4_ring/zigzag.py:1-18): a sequence of N tokens is cut into 2S chunks
// of h = N/(2S) rows; rank r holds chunk r then chunk 2S-1-r.  For packed
// sequences every sequence is sharded on its own, and the local shards are
// packed in sequence order, so local_cu[j] = full_cu[j] / S.
//
// All kernels are pure byte movement (HBM-bound): one output row per loop trip,
// copied with the widest vector (16/8/4/2/1 bytes) that the row size and the
// pointers allow, four vectors per thread in flight, grid sized to a multiple of the SM
// count.
#include "common.cuh"

namespace fa4cp {
namespace {

constexpr int kThreads = 256;

// One row: each thread loads up to kUnroll vectors before it stores any, so that enough
// bytes are in flight per SM to cover HBM latency (a load-then-store loop keeps one vector per
// thread in flight: 78% of the copy bandwidth measured on 8 KB rows).
constexpr int kUnroll = 4;

template <typename V>
struct Copier {
  __device__ __forceinline__ static void row(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                                             int64_t row_bytes) {
    const V* __restrict__ s = reinterpret_cast<const V*>(src);
    V* __restrict__ d = reinterpret_cast<V*>(dst);
    const int64_t n = row_bytes / int64_t(sizeof(V));
    for (int64_t i0 = threadIdx.x; i0 < n; i0 += int64_t(kUnroll) * blockDim.x) {
      V v[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int64_t i = i0 + int64_t(u) * blockDim.x;
        if (i < n) v[u] = s[i];
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int64_t i = i0 + int64_t(u) * blockDim.x;
        if (i < n) d[i] = v[u];
      }
    }
  }
};

// Largest j with cu[j] <= x (cu ascending, cu[0] = 0, x < cu[nseq]) scaled by `div`.
__device__ __forceinline__ int find_seq(const int32_t* __restrict__ cu, int nseq, int64_t x,
                                       int div) {
  int lo = 0, hi = nseq - 1;
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (int64_t(cu[mid] / div) <= x) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// out[local row] = x[full row] for rank `rank`.
template <typename V>
__global__ void __launch_bounds__(kThreads) zigzag_shard_kernel(
    const uint8_t* __restrict__ x, uint8_t* __restrict__ out, const int32_t* __restrict__ full_cu,
    int nseq, int64_t total_full, int rank, int S, int64_t row_bytes) {
  const int64_t total_local = total_full / S;
  for (int64_t r = blockIdx.x; r < total_local; r += gridDim.x) {
    int64_t seq_start = 0, n = total_full;
    if (full_cu != nullptr) {
      int j = find_seq(full_cu, nseq, r, S);
      seq_start = full_cu[j];
      n = int64_t(full_cu[j + 1]) - full_cu[j];
    }
    const int64_t h = n / (2 * S);
    const int64_t o = r - seq_start / S;  // offset inside this sequence's local shard
    const int64_t src = seq_start + (o < h ? int64_t(rank) * h + o : int64_t(2 * S - 1 - rank) * h + (o - h));
    Copier<V>::row(x + src * row_bytes, out + r * row_bytes, row_bytes);
  }
}

struct ShardPtrs {
  const uint8_t* p[64];
};

// out[full row] = shards[rank][local row].
template <typename V>
__global__ void __launch_bounds__(kThreads) zigzag_unshard_kernel(
    ShardPtrs shards, uint8_t* __restrict__ out, const int32_t* __restrict__ full_cu, int nseq,
    int64_t total_full, int S, int64_t row_bytes) {
  for (int64_t R = blockIdx.x; R < total_full; R += gridDim.x) {
    int64_t seq_start = 0, n = total_full;
    if (full_cu != nullptr) {
      int j = find_seq(full_cu, nseq, R, 1);
      seq_start = full_cu[j];
      n = int64_t(full_cu[j + 1]) - full_cu[j];
    }
    const int64_t h = n / (2 * S);
    const int64_t o = R - seq_start;
    const int64_t c = o / h, w = o - c * h;
    const int rank = c < S ? int(c) : int(2 * S - 1 - c);
    const int64_t local = seq_start / S + (c < S ? w : h + w);
    Copier<V>::row(shards.p[rank] + local * row_bytes, out + R * row_bytes, row_bytes);
  }
}

__global__ void half_index_kernel(const int32_t* __restrict__ cu, int nseq, int64_t half_total,
                                  int front, int64_t* __restrict__ out) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < half_total;
       i += int64_t(gridDim.x) * blockDim.x) {
    // half_cu = cu / 2 describes the packed half tensor
    int lo = 0, hi = nseq - 1;
    while (lo < hi) {
      int mid = (lo + hi + 1) >> 1;
      if (int64_t(cu[mid] / 2) <= i) lo = mid; else hi = mid - 1;
    }
    const int64_t s = cu[lo], e = cu[lo + 1];
    const int64_t o = i - s / 2;
    out[i] = (front ? s : (s + e) / 2) + o;
  }
}

__global__ void local_cu_kernel(const int32_t* __restrict__ full_cu, int n, int S,
                                int32_t* __restrict__ local_cu) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) local_cu[i] = full_cu[i] / S;
}

// GDN context-parallel index metadata (the reference's fa4_ring/gdn_cp/metadata.py:48-96):
// restore[n] = slot of natural token n in the rank-major all-gather [rank0 | rank1 | ...]
// (each rank's part L = total / S rows); extract[i] = natural position of local token i of
// rank `rank`.  Sequence j: natural rows [full_cu[j], full_cu[j+1]), local rows
// [full_cu[j] / S, full_cu[j+1] / S), h = N_j / (2S); local position p < h is chunk `rank`,
// p >= h chunk 2S-1-rank.
__global__ void gdn_indices_kernel(const int32_t* __restrict__ full_cu, int nseq, int S, int rank,
                                   int64_t total, int64_t* __restrict__ restore,
                                   int64_t* __restrict__ extract) {
  const int64_t L = total / S;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t n = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; n < total; n += stride) {
    if (restore != nullptr) {
      const int j = find_seq(full_cu, nseq, n, 1);
      const int64_t a = full_cu[j], h = (int64_t(full_cu[j + 1]) - a) / (2 * S);
      const int64_t o = n - a, c = o / h, q = o - c * h;
      const int64_t r = c < S ? c : 2 * S - 1 - c;
      const int64_t p = c < S ? q : h + q;
      restore[n] = r * L + a / S + p;
    }
    if (extract != nullptr && n < L) {
      const int j = find_seq(full_cu, nseq, n, S);
      const int64_t a = full_cu[j], h = (int64_t(full_cu[j + 1]) - a) / (2 * S);
      const int64_t p = n - a / S;
      extract[n] = a + (p < h ? int64_t(rank) * h + p : (2 * S - 1 - int64_t(rank)) * h + (p - h));
    }
  }
}

int num_sms() {
  static int sms = 0;
  if (sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  return sms;
}

int vec_width(int64_t row_bytes, std::initializer_list<const void*> ptrs) {
  uintptr_t a = 0;
  for (const void* p : ptrs) a |= reinterpret_cast<uintptr_t>(p);
  for (int w : {16, 8, 4, 2}) {
    if (row_bytes % w == 0 && (a % w) == 0) return w;
  }
  return 1;
}

int64_t grid_rows(int64_t rows) {
  const int64_t cap = int64_t(num_sms()) * 16;  // 16 x 256-thread CTAs resident per SM
  return rows < cap ? (rows > 0 ? rows : 1) : cap;
}

}  // namespace
}  // namespace fa4cp

using namespace fa4cp;

extern "C" int fa4cp_zigzag_shard(const void* x, void* out, const int32_t* full_cu, int32_t nseq,
                                  int64_t total_full, int32_t cp_rank, int32_t cp_size,
                                  int64_t row_bytes, void* stream) {
  FA4CP_CHECK_ARG(cp_size >= 1 && cp_size <= 64, "cp_size must be in [1, 64], got %d", cp_size);
  FA4CP_CHECK_ARG(cp_rank >= 0 && cp_rank < cp_size, "cp_rank %d out of range", cp_rank);
  FA4CP_CHECK_ARG(total_full >= 0 && row_bytes > 0, "bad sizes");
  FA4CP_CHECK_ARG(full_cu != nullptr ? nseq >= 1 : total_full % (2 * cp_size) == 0,
                  "seqlen %lld must be divisible by 2*cp_size=%d", (long long)total_full,
                  2 * cp_size);
  FA4CP_CHECK_ARG(total_full % cp_size == 0, "total rows not divisible by cp_size");
  if (total_full == 0) return FA4CP_OK;
  FA4CP_CHECK_ARG(x != nullptr && out != nullptr, "null tensor pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t rows = total_full / cp_size;
  dim3 grid(unsigned(grid_rows(rows)));
  auto* xs = static_cast<const uint8_t*>(x);
  auto* os = static_cast<uint8_t*>(out);
  switch (vec_width(row_bytes, {x, out})) {
    case 16: zigzag_shard_kernel<uint4><<<grid, kThreads, 0, st>>>(xs, os, full_cu, nseq, total_full, cp_rank, cp_size, row_bytes); break;
    case 8: zigzag_shard_kernel<uint2><<<grid, kThreads, 0, st>>>(xs, os, full_cu, nseq, total_full, cp_rank, cp_size, row_bytes); break;
    case 4: zigzag_shard_kernel<uint32_t><<<grid, kThreads, 0, st>>>(xs, os, full_cu, nseq, total_full, cp_rank, cp_size, row_bytes); break;
    case 2: zigzag_shard_kernel<uint16_t><<<grid, kThreads, 0, st>>>(xs, os, full_cu, nseq, total_full, cp_rank, cp_size, row_bytes); break;
    default: zigzag_shard_kernel<uint8_t><<<grid, kThreads, 0, st>>>(xs, os, full_cu, nseq, total_full, cp_rank, cp_size, row_bytes); break;
  }
  return check_launch("zigzag_shard");
}

extern "C" int fa4cp_zigzag_unshard(const void* const* shards, void* out, const int32_t* full_cu,
                                    int32_t nseq, int64_t total_full, int32_t cp_size,
                                    int64_t row_bytes, void* stream) {
  FA4CP_CHECK_ARG(cp_size >= 1 && cp_size <= 64, "cp_size must be in [1, 64], got %d", cp_size);
  FA4CP_CHECK_ARG(shards != nullptr, "shards must be a host array of cp_size pointers");
  FA4CP_CHECK_ARG(total_full >= 0 && row_bytes > 0, "bad sizes");
  FA4CP_CHECK_ARG(full_cu != nullptr ? nseq >= 1 : total_full % (2 * cp_size) == 0,
                  "seqlen %lld must be divisible by 2*cp_size=%d", (long long)total_full,
                  2 * cp_size);
  if (total_full == 0) return FA4CP_OK;
  ShardPtrs sp{};
  uintptr_t a = reinterpret_cast<uintptr_t>(out);
  for (int i = 0; i < cp_size; ++i) {
    FA4CP_CHECK_ARG(shards[i] != nullptr, "shard %d is NULL", i);
    sp.p[i] = static_cast<const uint8_t*>(shards[i]);
    a |= reinterpret_cast<uintptr_t>(shards[i]);
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  dim3 grid(unsigned(grid_rows(total_full)));
  auto* os = static_cast<uint8_t*>(out);
  int w = vec_width(row_bytes, {reinterpret_cast<const void*>(a)});
  switch (w) {
    case 16: zigzag_unshard_kernel<uint4><<<grid, kThreads, 0, st>>>(sp, os, full_cu, nseq, total_full, cp_size, row_bytes); break;
    case 8: zigzag_unshard_kernel<uint2><<<grid, kThreads, 0, st>>>(sp, os, full_cu, nseq, total_full, cp_size, row_bytes); break;
    case 4: zigzag_unshard_kernel<uint32_t><<<grid, kThreads, 0, st>>>(sp, os, full_cu, nseq, total_full, cp_size, row_bytes); break;
    case 2: zigzag_unshard_kernel<uint16_t><<<grid, kThreads, 0, st>>>(sp, os, full_cu, nseq, total_full, cp_size, row_bytes); break;
    default: zigzag_unshard_kernel<uint8_t><<<grid, kThreads, 0, st>>>(sp, os, full_cu, nseq, total_full, cp_size, row_bytes); break;
  }
  return check_launch("zigzag_unshard");
}

extern "C" int fa4cp_half_index(const int32_t* cu, int32_t nseq, int64_t total, int32_t front,
                                int64_t* out_idx, void* stream) {
  FA4CP_CHECK_ARG(nseq >= 1 && cu != nullptr, "cu must describe at least one sequence");
  FA4CP_CHECK_ARG(total >= 0 && total % 2 == 0, "each local sequence length must be even (zig-zag)");
  if (total == 0) return FA4CP_OK;
  const int64_t half = total / 2;
  const int threads = 256;
  int64_t blocks = (half + threads - 1) / threads;
  if (blocks > int64_t(num_sms()) * 8) blocks = int64_t(num_sms()) * 8;
  half_index_kernel<<<unsigned(blocks), threads, 0, static_cast<cudaStream_t>(stream)>>>(
      cu, nseq, half, front, out_idx);
  return check_launch("half_index");
}

extern "C" int fa4cp_gdn_cp_indices(const int32_t* full_cu, int32_t nseq, int32_t cp_size,
                                    int32_t cp_rank, int64_t total, int64_t* restore_perm,
                                    int64_t* extract_idx, void* stream) {
  FA4CP_CHECK_ARG(nseq >= 1 && full_cu != nullptr, "full_cu must describe at least one sequence");
  FA4CP_CHECK_ARG(cp_size >= 1 && cp_rank >= 0 && cp_rank < cp_size, "bad cp rank %d of %d",
                  cp_rank, cp_size);
  FA4CP_CHECK_ARG(total >= 0 && total % (2 * int64_t(cp_size)) == 0,
                  "total %lld is not a multiple of 2*cp_size", static_cast<long long>(total));
  if (total == 0 || (restore_perm == nullptr && extract_idx == nullptr)) return FA4CP_OK;
  const int threads = 256;
  int64_t blocks = (total + threads - 1) / threads;
  if (blocks > int64_t(num_sms()) * 8) blocks = int64_t(num_sms()) * 8;
  gdn_indices_kernel<<<unsigned(blocks), threads, 0, static_cast<cudaStream_t>(stream)>>>(
      full_cu, nseq, cp_size, cp_rank, total, restore_perm, extract_idx);
  return check_launch("gdn_cp_indices");
}

extern "C" int fa4cp_local_cu(const int32_t* full_cu, int32_t nseq, int32_t cp_size,
                              int32_t* local_cu, void* stream) {
  FA4CP_CHECK_ARG(nseq >= 0 && full_cu != nullptr && local_cu != nullptr, "bad arguments");
  FA4CP_CHECK_ARG(cp_size >= 1, "cp_size must be >= 1");
  const int n = nseq + 1;
  local_cu_kernel<<<(n + 127) / 128, 128, 0, static_cast<cudaStream_t>(stream)>>>(full_cu, n,
                                                                                 cp_size, local_cu);
  return check_launch("local_cu");
}
