// Online-softmax LSE merge kernels (natural-log LSE, fp32 math).
//
// Restates the math of the reference's merge (tests/test_algorithm_cpu.py:51-59):
//   m = max(s_a, s_b); w_a = e^(s_a - m); w_b = e^(s_b - m)
//   v = (v_a w_a + v_b w_b) / (w_a + w_b);  s = m + log(w_a + w_b)
// computed with base-2 hardware exp/log on LSE values converted by log2(e).
//
// HBM-bound.  One thread owns one 16-byte vector of one (row, head): it reads the
// two LSE words (broadcast within the group of threads of that (row, head)), the
// two value vectors, and writes one vector (+ the LSE from the group leader).
// A partial whose LSE is -inf is never read (a back-half-only step leaves the
// front rows' values undefined); a row where both LSEs are -inf gets zeros and -inf.
#include "common.cuh"

namespace fa4cp {
namespace {

template <typename T> struct Vec;
template <> struct Vec<__nv_bfloat16> { static constexpr int N = 8; };
template <> struct Vec<__half> { static constexpr int N = 8; };
template <> struct Vec<float> { static constexpr int N = 4; };

__device__ __forceinline__ void unpack(const uint4& u, float* f, __nv_bfloat16*) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}
__device__ __forceinline__ void unpack(const uint4& u, float* f, __half*) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
    float2 t = __half22float2(h);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}
__device__ __forceinline__ void unpack(const uint4& u, float* f, float*) {
  f[0] = __uint_as_float(u.x); f[1] = __uint_as_float(u.y);
  f[2] = __uint_as_float(u.z); f[3] = __uint_as_float(u.w);
}
__device__ __forceinline__ uint4 pack(const float* f, __nv_bfloat16*) {
  return make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]),
                    pack_bf16x2(f[6], f[7]));
}
__device__ __forceinline__ uint4 pack(const float* f, __half*) {
  return make_uint4(pack_f16x2(f[0], f[1]), pack_f16x2(f[2], f[3]), pack_f16x2(f[4], f[5]),
                    pack_f16x2(f[6], f[7]));
}
__device__ __forceinline__ uint4 pack(const float* f, float*) {
  return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]),
                    __float_as_uint(f[3]));
}

constexpr float kNegInf = -__builtin_huge_valf();

// Value pass of the in-place merge.  It only reads the LSE words; they are
// rewritten by merge_inplace_lse_kernel afterwards (a thread of the same
// (row, head) group may run in another CTA, so the update cannot share a pass).
template <typename T>
__global__ void __launch_bounds__(256) merge_inplace_kernel(
    uint4* __restrict__ v, const float* __restrict__ s, const uint4* __restrict__ vo,
    const float* __restrict__ so, int64_t num_rh, int vecs_per_head) {
  constexpr int N = Vec<T>::N;
  const int64_t total = num_rh * vecs_per_head;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t rh = i / vecs_per_head;
    const float sa = s[rh], sb = so[rh];
    if (sb == kNegInf) {                  // partial covers nothing here: identity, or zeros
      if (sa == kNegInf) {                // when neither covers the row (the reference's
        float z[N];                       // clamped denominator gives 0)
#pragma unroll
        for (int e = 0; e < N; ++e) z[e] = 0.f;
        v[i] = pack(z, (T*)nullptr);
      }
      continue;
    }
    float fa[N], fb[N];
    unpack(vo[i], fb, (T*)nullptr);
    if (sa == kNegInf) {                   // accumulator empty: take the partial
#pragma unroll
      for (int e = 0; e < N; ++e) fa[e] = fb[e];
    } else {
      unpack(v[i], fa, (T*)nullptr);
      const float m = fmaxf(sa, sb);
      const float wa = ex2_approx((sa - m) * kLog2e);
      const float wb = ex2_approx((sb - m) * kLog2e);
      const float inv = 1.0f / (wa + wb);
      const float ca = wa * inv, cb = wb * inv;
#pragma unroll
      for (int e = 0; e < N; ++e) fa[e] = fa[e] * ca + fb[e] * cb;
    }
    v[i] = pack(fa, (T*)nullptr);
  }
}

// Single-pass in-place merge when a head holds 2^LOG <= 32 vectors: the flat vector index is
// walked in warp-sized chunks, so the vectors of one (row, head) lie in one warp; after a
// __syncwarp (every lane of the group has read the old LSE) the group's first lane writes the
// merged LSE.  Shifts replace the 64-bit division of the generic form, and each warp takes
// U chunks per trip with all their loads (LSEs and vectors) issued together, so that U
// independent DRAM round trips are in flight per thread.
template <typename T, int LOG>
__global__ void __launch_bounds__(256) merge_inplace_fused_kernel(
    uint4* __restrict__ v, float* __restrict__ s, const uint4* __restrict__ vo,
    const float* __restrict__ so, int64_t total) {
  static_assert(LOG >= 0 && LOG <= 5, "a head's vectors must fit in one warp");
  constexpr int N = Vec<T>::N, VPH = 1 << LOG, U = 4;
  const int lane = threadIdx.x & 31;
  const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t warps = (int64_t(gridDim.x) * blockDim.x) >> 5;
  for (int64_t base = warp * 32 * U; base < total; base += warps * 32 * U) {  // warp-uniform
    // every load of the trip is issued at once -- LSEs and vectors -- so one DRAM round trip
    // is in flight, not two dependent ones (gating the vector loads on finite LSEs measured
    // 73% of the copy bandwidth); a -inf operand's vector is loaded but never used
    float sa[U], sb[U];
    uint4 ra[U], rb[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t i = base + u * 32 + lane;
      sa[u] = sb[u] = kNegInf;
      if (i < total) {
        sa[u] = s[i >> LOG];
        sb[u] = so[i >> LOG];
        rb[u] = vo[i];
        ra[u] = v[i];
      }
    }
    float s_new[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t i = base + u * 32 + lane;
      s_new[u] = sa[u];
      if (i >= total) continue;
      float fa[N];
      if (sb[u] == kNegInf) {
        if (sa[u] != kNegInf) continue;  // a partial covering nothing is the identity
#pragma unroll
        for (int e = 0; e < N; ++e) fa[e] = 0.f;  // neither covers the row: zeros, as the
      } else {                                      // reference's clamped denominator gives
        float fb[N];
        unpack(rb[u], fb, (T*)nullptr);
        if (sa[u] == kNegInf) {  // accumulator empty: take the partial
#pragma unroll
          for (int e = 0; e < N; ++e) fa[e] = fb[e];
          s_new[u] = sb[u];
        } else {
          unpack(ra[u], fa, (T*)nullptr);
          const float m = fmaxf(sa[u], sb[u]);
          const float wa = ex2_approx((sa[u] - m) * kLog2e);
          const float wb = ex2_approx((sb[u] - m) * kLog2e);
          const float inv = 1.0f / (wa + wb);
          const float ca = wa * inv, cb = wb * inv;
#pragma unroll
          for (int e = 0; e < N; ++e) fa[e] = fa[e] * ca + fb[e] * cb;
          s_new[u] = m + lg2_approx(wa + wb) * kLn2;
        }
      }
      v[i] = pack(fa, (T*)nullptr);
    }
    __syncwarp();
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t i = base + u * 32 + lane;
      if (i < total && sb[u] != kNegInf && (lane & (VPH - 1)) == 0) s[i >> LOG] = s_new[u];
    }
  }
}

// LSE pass of the in-place merge: s <- logaddexp(s, s_other).
__global__ void __launch_bounds__(256) merge_inplace_lse_kernel(float* __restrict__ s,
                                                               const float* __restrict__ so,
                                                               int64_t num_rh) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < num_rh;
       i += int64_t(gridDim.x) * blockDim.x) {
    const float sa = s[i], sb = so[i];
    if (sb == kNegInf) continue;
    if (sa == kNegInf) {
      s[i] = sb;
      continue;
    }
    const float m = fmaxf(sa, sb);
    const float wa = ex2_approx((sa - m) * kLog2e);
    const float wb = ex2_approx((sb - m) * kLog2e);
    s[i] = m + lg2_approx(wa + wb) * kLn2;
  }
}

struct StatePtrs {
  const uint4* v[32];
  const float* s[32];
};

template <typename T>
__global__ void __launch_bounds__(256) merge_states_kernel(StatePtrs ptrs, int k,
                                                          uint4* __restrict__ vout,
                                                          float* __restrict__ sout, int64_t num_rh,
                                                          int vecs_per_head) {
  constexpr int N = Vec<T>::N;
  const int64_t total = num_rh * vecs_per_head;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t rh = i / vecs_per_head;
    const int c = int(i - rh * vecs_per_head);
    float m = kNegInf;
    for (int j = 0; j < k; ++j) m = fmaxf(m, ptrs.s[j][rh]);
    float acc[N];
#pragma unroll
    for (int e = 0; e < N; ++e) acc[e] = 0.f;
    float den = 0.f;
    if (m != kNegInf) {
      for (int j = 0; j < k; ++j) {
        const float sj = ptrs.s[j][rh];
        if (sj == kNegInf) continue;
        const float w = ex2_approx((sj - m) * kLog2e);
        float f[N];
        unpack(ptrs.v[j][i], f, (T*)nullptr);
#pragma unroll
        for (int e = 0; e < N; ++e) acc[e] += f[e] * w;
        den += w;
      }
      const float inv = 1.0f / den;
#pragma unroll
      for (int e = 0; e < N; ++e) acc[e] *= inv;
    }
    vout[i] = pack(acc, (T*)nullptr);
    if (sout != nullptr && c == 0) sout[rh] = (m == kNegInf) ? kNegInf : m + lg2_approx(den) * kLn2;
  }
}

__global__ void fill_kernel(float* __restrict__ p, int64_t n, float value) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n;
       i += int64_t(gridDim.x) * blockDim.x)
    p[i] = value;
}

int sm_count() {
  static int sms = 0;
  if (sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  return sms;
}

unsigned grid_for(int64_t work) {
  int64_t b = (work + 255) / 256;
  const int64_t cap = int64_t(sm_count()) * 8;
  if (b > cap) b = cap;
  return unsigned(b > 0 ? b : 1);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace fa4cp

using namespace fa4cp;

extern "C" int fa4cp_merge_state_inplace(void* v, float* s, const void* v_other,
                                         const float* s_other, int64_t num_rows,
                                         int32_t num_heads, int32_t head_dim, int32_t dtype,
                                         void* stream) {
  FA4CP_CHECK_ARG(num_rows >= 0 && num_heads > 0 && head_dim > 0, "bad sizes");
  FA4CP_CHECK_ARG(dtype == FA4CP_DTYPE_BF16 || dtype == FA4CP_DTYPE_F16 || dtype == FA4CP_DTYPE_F32,
                  "merge supports f16, bf16, f32 values (got dtype %d)", dtype);
  const int per = (dtype == FA4CP_DTYPE_F32) ? 4 : 8;
  FA4CP_CHECK_ARG(head_dim % per == 0, "head_dim %d must be a multiple of %d", head_dim, per);
  if (num_rows == 0) return FA4CP_OK;
  FA4CP_CHECK_ARG(aligned16(v) && aligned16(v_other), "value tensors must be 16-byte aligned");
  const int64_t rh = num_rows * num_heads;
  const int vph = head_dim / per;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned g = grid_for(rh * vph);
  auto* vv = static_cast<uint4*>(v);
  auto* vo = static_cast<const uint4*>(v_other);
  if ((vph & (vph - 1)) == 0 && vph <= 32) {  // one pass (the common head_dim 64 / 128 / 256)
    int lg = 0;
    while ((1 << lg) < vph) ++lg;
    const int64_t total = rh * vph;
#define FA4CP_MERGE_FUSED(T)                                                                     \
    switch (lg) {                                                                              \
      case 0: merge_inplace_fused_kernel<T, 0><<<g, 256, 0, st>>>(vv, s, vo, s_other, total); break; \
      case 1: merge_inplace_fused_kernel<T, 1><<<g, 256, 0, st>>>(vv, s, vo, s_other, total); break; \
      case 2: merge_inplace_fused_kernel<T, 2><<<g, 256, 0, st>>>(vv, s, vo, s_other, total); break; \
      case 3: merge_inplace_fused_kernel<T, 3><<<g, 256, 0, st>>>(vv, s, vo, s_other, total); break; \
      case 4: merge_inplace_fused_kernel<T, 4><<<g, 256, 0, st>>>(vv, s, vo, s_other, total); break; \
      default: merge_inplace_fused_kernel<T, 5><<<g, 256, 0, st>>>(vv, s, vo, s_other, total); break; \
    }
    if (dtype == FA4CP_DTYPE_BF16) {
      FA4CP_MERGE_FUSED(__nv_bfloat16)
    } else if (dtype == FA4CP_DTYPE_F16) {
      FA4CP_MERGE_FUSED(__half)
    } else {
      FA4CP_MERGE_FUSED(float)
    }
#undef FA4CP_MERGE_FUSED
    return check_launch("merge_state_inplace");
  }
  if (dtype == FA4CP_DTYPE_BF16)
    merge_inplace_kernel<__nv_bfloat16><<<g, 256, 0, st>>>(vv, s, vo, s_other, rh, vph);
  else if (dtype == FA4CP_DTYPE_F16)
    merge_inplace_kernel<__half><<<g, 256, 0, st>>>(vv, s, vo, s_other, rh, vph);
  else
    merge_inplace_kernel<float><<<g, 256, 0, st>>>(vv, s, vo, s_other, rh, vph);
  int rc = check_launch("merge_state_inplace");
  if (rc) return rc;
  merge_inplace_lse_kernel<<<grid_for(rh), 256, 0, st>>>(s, s_other, rh);
  return check_launch("merge_state_inplace(lse)");
}

extern "C" int fa4cp_merge_states(const void* const* v_ptrs, const float* const* s_ptrs,
                                  int32_t num_states, void* v_out, float* s_out, int64_t num_rows,
                                  int32_t num_heads, int32_t head_dim, int32_t dtype,
                                  void* stream) {
  FA4CP_CHECK_ARG(num_states >= 1 && num_states <= 32, "num_states must be in [1, 32], got %d",
                  num_states);
  FA4CP_CHECK_ARG(v_ptrs != nullptr && s_ptrs != nullptr, "pointer arrays must not be NULL");
  FA4CP_CHECK_ARG(num_rows >= 0 && num_heads > 0 && head_dim > 0, "bad sizes");
  FA4CP_CHECK_ARG(dtype == FA4CP_DTYPE_BF16 || dtype == FA4CP_DTYPE_F16 || dtype == FA4CP_DTYPE_F32,
                  "merge supports f16, bf16, f32 values (got dtype %d)", dtype);
  const int per = (dtype == FA4CP_DTYPE_F32) ? 4 : 8;
  FA4CP_CHECK_ARG(head_dim % per == 0, "head_dim %d must be a multiple of %d", head_dim, per);
  if (num_rows == 0) return FA4CP_OK;
  StatePtrs p{};
  for (int i = 0; i < num_states; ++i) {
    FA4CP_CHECK_ARG(v_ptrs[i] != nullptr && s_ptrs[i] != nullptr, "state %d is NULL", i);
    FA4CP_CHECK_ARG(aligned16(v_ptrs[i]), "state %d values must be 16-byte aligned", i);
    p.v[i] = static_cast<const uint4*>(v_ptrs[i]);
    p.s[i] = s_ptrs[i];
  }
  FA4CP_CHECK_ARG(aligned16(v_out), "output must be 16-byte aligned");
  const int64_t rh = num_rows * num_heads;
  const int vph = head_dim / per;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned g = grid_for(rh * vph);
  auto* vo = static_cast<uint4*>(v_out);
  if (dtype == FA4CP_DTYPE_BF16)
    merge_states_kernel<__nv_bfloat16><<<g, 256, 0, st>>>(p, num_states, vo, s_out, rh, vph);
  else if (dtype == FA4CP_DTYPE_F16)
    merge_states_kernel<__half><<<g, 256, 0, st>>>(p, num_states, vo, s_out, rh, vph);
  else
    merge_states_kernel<float><<<g, 256, 0, st>>>(p, num_states, vo, s_out, rh, vph);
  return check_launch("merge_states");
}

extern "C" int fa4cp_fill_f32(float* dst, int64_t n, float value, void* stream) {
  FA4CP_CHECK_ARG(n >= 0, "bad size");
  if (n == 0) return FA4CP_OK;
  FA4CP_CHECK_ARG(dst != nullptr, "dst is NULL");
  fill_kernel<<<grid_for(n), 256, 0, static_cast<cudaStream_t>(stream)>>>(dst, n, value);
  return check_launch("fill_f32");
}
