// FP8 e4m3 conversion kernels (HBM-bound).
//
// * fa4cp_dequant_e4m3: e4m3 [rows, heads, dim] x descale[heads] -> bf16, used to feed
//   e4m3 K/V into the bf16 attention kernel when Q is bf16 (a tcgen05 kind::f16 MMA
//   takes one operand type for A and B).
// * fa4cp_quantize_e4m3: per-tensor quantisation scale = amax / 448, q = x / scale
//   (the recipe of the FP8 configs: each rank quantises its own shard and the K/V
//   descales are all-gathered), in two passes: an amax reduction into *scale, then a
//   cast that reads the scale.
#include "common.cuh"

namespace fa4cp {
namespace {

constexpr float kE4M3Max = 448.0f;

// 16 e4m3 bytes -> 16 bf16 (two uint4), scaled by s
__global__ void __launch_bounds__(256) dequant_kernel(const uint4* __restrict__ x,
                                                      const float* __restrict__ descale,
                                                      uint4* __restrict__ out, int64_t n16,
                                                      int vec_per_head, int heads) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n16;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int h = int((i / vec_per_head) % heads);
    const float s = descale ? descale[h] : 1.0f;
    const uint4 v = x[i];
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    uint32_t o[8];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      // two e4m3 pairs -> float2 each, via the hardware e4m3x2 -> f16x2 conversion
      uint32_t h01, h23;
      const uint16_t lo = uint16_t(w[k] & 0xFFFF), hi = uint16_t(w[k] >> 16);
      asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h01) : "h"(lo));
      asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h23) : "h"(hi));
      const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&h01));
      const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&h23));
      o[2 * k] = pack_bf16x2(a.x * s, a.y * s);
      o[2 * k + 1] = pack_bf16x2(b.x * s, b.y * s);
    }
    out[2 * i] = make_uint4(o[0], o[1], o[2], o[3]);
    out[2 * i + 1] = make_uint4(o[4], o[5], o[6], o[7]);
  }
}

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }

// amax over the tensor -> scale = amax / 448 (stored as float bits via atomicMax on
// the non-negative float's integer image, which orders like the float)
template <typename T>
__global__ void __launch_bounds__(256) amax_kernel(const T* __restrict__ x, int64_t n,
                                                   unsigned int* __restrict__ amax_bits) {
  float m = 0.f;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n;
       i += int64_t(gridDim.x) * blockDim.x)
    m = fmaxf(m, fabsf(to_f(x[i])));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  __shared__ float red[8];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < int(blockDim.x >> 5); ++w) m = fmaxf(m, red[w]);
    atomicMax(amax_bits, __float_as_uint(m));
  }
}

__global__ void finish_scale_kernel(unsigned int* amax_bits_scale) {
  const float amax = __uint_as_float(*amax_bits_scale);
  const float scale = amax > 0.f ? amax / kE4M3Max : 1.0f;
  *reinterpret_cast<float*>(amax_bits_scale) = scale;
}

template <typename T>
__global__ void __launch_bounds__(256) quant_kernel(const T* __restrict__ x, int64_t n,
                                                    const float* __restrict__ scale,
                                                    uint16_t* __restrict__ out2) {
  const float s = *scale;
  const int64_t n2 = n / 2;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n2;
       i += int64_t(gridDim.x) * blockDim.x) {
    const float a = to_f(x[2 * i]) / s, b = to_f(x[2 * i + 1]) / s;  // IEEE division
    uint16_t r;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(b), "f"(a));
    out2[i] = r;
  }
}

int sms() {
  static int s = 0;
  if (s == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&s, cudaDevAttrMultiProcessorCount, dev);
    if (s <= 0) s = 148;
  }
  return s;
}

unsigned grid_for(int64_t work) {
  int64_t b = (work + 255) / 256;
  const int64_t cap = int64_t(sms()) * 8;
  if (b > cap) b = cap;
  return unsigned(b > 0 ? b : 1);
}

}  // namespace

// shared with attn_fwd_sm100.cu (the kv8 entry point dequantises through it)
int launch_dequant_e4m3(const void* x, const float* descale, void* out, int64_t rows, int heads,
                        int dim, cudaStream_t st) {
  FA4CP_CHECK_ARG(rows >= 0 && heads > 0 && dim > 0 && dim % 16 == 0,
                  "dequant needs dim %% 16 == 0 (got %d)", dim);
  FA4CP_CHECK_ARG((reinterpret_cast<uintptr_t>(x) & 15u) == 0 &&
                      (reinterpret_cast<uintptr_t>(out) & 15u) == 0,
                  "dequant tensors must be 16-byte aligned");
  const int64_t n16 = rows * heads * int64_t(dim) / 16;
  if (n16 == 0) return FA4CP_OK;
  dequant_kernel<<<grid_for(n16), 256, 0, st>>>(static_cast<const uint4*>(x), descale,
                                                 static_cast<uint4*>(out), n16, dim / 16, heads);
  return check_launch("dequant_e4m3");
}

}  // namespace fa4cp

using namespace fa4cp;

extern "C" int fa4cp_dequant_e4m3(const void* x, const float* descale, void* out, int64_t rows,
                                  int32_t heads, int32_t dim, void* stream) {
  return launch_dequant_e4m3(x, descale, out, rows, heads, dim, static_cast<cudaStream_t>(stream));
}

extern "C" int fa4cp_quantize_e4m3(const void* x, int32_t dtype, int64_t n, void* out,
                                   float* scale, void* stream) {
  FA4CP_CHECK_ARG(n >= 0 && n % 2 == 0, "element count must be even");
  FA4CP_CHECK_ARG(scale != nullptr, "scale must not be NULL");
  FA4CP_CHECK_ARG(dtype == FA4CP_DTYPE_BF16 || dtype == FA4CP_DTYPE_F16 || dtype == FA4CP_DTYPE_F32,
                  "quantize supports f16, bf16, f32 inputs");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  FA4CP_CHECK_CUDA(cudaMemsetAsync(scale, 0, sizeof(float), st));
  auto* bits = reinterpret_cast<unsigned int*>(scale);
  const unsigned g = grid_for(n);
  if (n > 0) {
    if (dtype == FA4CP_DTYPE_BF16)
      amax_kernel<__nv_bfloat16><<<g, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(x), n, bits);
    else if (dtype == FA4CP_DTYPE_F16)
      amax_kernel<__half><<<g, 256, 0, st>>>(static_cast<const __half*>(x), n, bits);
    else
      amax_kernel<float><<<g, 256, 0, st>>>(static_cast<const float*>(x), n, bits);
  }
  finish_scale_kernel<<<1, 1, 0, st>>>(bits);
  if (n > 0) {
    auto* o = static_cast<uint16_t*>(out);
    if (dtype == FA4CP_DTYPE_BF16)
      quant_kernel<__nv_bfloat16><<<g, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(x), n, scale, o);
    else if (dtype == FA4CP_DTYPE_F16)
      quant_kernel<__half><<<g, 256, 0, st>>>(static_cast<const __half*>(x), n, scale, o);
    else
      quant_kernel<float><<<g, 256, 0, st>>>(static_cast<const float*>(x), n, scale, o);
  }
  return check_launch("quantize_e4m3");
}
