// Shared device helpers for the sm_100a kernels of fa4cp_b200: error plumbing,
// mbarriers with bounded waits, TMA bulk-tensor loads, and tcgen05 (TMEM + UMMA)
// wrappers written directly in inline PTX.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/fa4cp_b200.h"

namespace fa4cp {

// ---------------------------------------------------------------------------
// host-side error reporting
// ---------------------------------------------------------------------------
void set_last_error(const char* fmt, ...);

#define FA4CP_CHECK_ARG(cond, ...)                 \
  do {                                             \
    if (!(cond)) {                                 \
      ::fa4cp::set_last_error(__VA_ARGS__);        \
      return FA4CP_ERR_INVALID;                    \
    }                                              \
  } while (0)

#define FA4CP_CHECK_CUDA(expr)                                                     \
  do {                                                                             \
    cudaError_t e_ = (expr);                                                       \
    if (e_ != cudaSuccess) {                                                       \
      ::fa4cp::set_last_error("%s failed: %s", #expr, cudaGetErrorString(e_));     \
      return FA4CP_ERR_CUDA;                                                       \
    }                                                                              \
  } while (0)

inline int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_error("%s launch failed: %s", what, cudaGetErrorString(e));
    return FA4CP_ERR_CUDA;
  }
  return FA4CP_OK;
}

// e4m3 [rows, heads, dim] x descale[heads] -> bf16 (convert.cu)
int launch_dequant_e4m3(const void* x, const float* descale, void* out, int64_t rows, int heads,
                        int dim, cudaStream_t st);

// SMs the persistent attention grid leaves free for concurrent kernels, for launches made by
// the calling host thread (attn_fwd_sm100.cu); 0 = use every SM
void set_sm_reserve(int n);

// fa4cp_ring_attn_fused with a general arrival-flag layout: slot s-1 is present once
// arrived[(s-1) * arrived_stride] >= arrived_base + s * arrived_step (attn_fwd_sm100.cu)
int ring_attn_fused_flags(const void* q, const void* k, const void* v, const void* slots_k,
                          const void* slots_v, int64_t slot_stride, void* out, float* lse,
                          const int32_t* cu, int32_t nseq, int32_t max_seqlen, int64_t total,
                          int32_t num_heads_q, int32_t num_heads_kv, int32_t head_dim,
                          int32_t dtype, float softmax_scale, const float* q_descale,
                          const float* k_descales, const float* v_descales, int32_t nranks,
                          int32_t rank, const uint32_t* arrived, uint32_t arrived_base,
                          int32_t arrived_stride, int32_t arrived_step, int32_t first_step,
                          int32_t accumulate, void* stream);

inline int elem_bytes(int dtype) {
  switch (dtype) {
    case FA4CP_DTYPE_F16: return 2;
    case FA4CP_DTYPE_BF16: return 2;
    case FA4CP_DTYPE_F32: return 4;
    case FA4CP_DTYPE_E4M3: return 1;
    default: return 0;
  }
}

// ---------------------------------------------------------------------------
// small device math (hardware instructions, no library sequences)
// ---------------------------------------------------------------------------
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float lg2_approx(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// ---------------------------------------------------------------------------
// shared-memory addresses, mbarriers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait on phase `parity` of an mbarrier.  Gives up after ~`kWaitLimitCycles`
// clock cycles, recording `code` in the device status word `*status` (first writer
// wins); gives up at once when another thread of the CTA (`*abort`) or another CTA
// (`*status`) already did.  Returns false on give-up.
constexpr long long kWaitLimitCycles = 4000000000LL;  // ~2 s at 1.9 GHz

__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort,
                                          int code, int* status) {
  if (mbar_try_wait(bar, parity)) return true;
  long long t0 = clock64();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 0) {
      if (*abort) return false;
      if (*reinterpret_cast<volatile int*>(status) != 0) {  // another CTA already gave up
        *abort = 1;
        return false;
      }
      if (clock64() - t0 > kWaitLimitCycles) {
        *abort = 1;
        atomicCAS(status, 0, code);
        return false;
      }
    }
  }
}

// Wait used only on the give-up path, for work this CTA itself already issued (TMA
// copies, MMAs): they always finish, and the CTA must not exit or free TMEM before they
// do.  It ignores the abort flags (which are set on this path) and is bounded by time
// alone; if even that runs out it records `code` and returns false.
__device__ __forceinline__ bool mbar_wait_drain(uint32_t bar, uint32_t parity, int code,
                                                int* status) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 0 && clock64() - t0 > kWaitLimitCycles) {
      atomicCAS(status, 0, code);
      return false;
    }
  }
}

// ---------------------------------------------------------------------------
// TMA (bulk tensor copies, global -> shared), no multicast
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const void* tmap, int c0, int c1, int c2,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(c0), "r"(c1), "r"(c2), "r"(bar)
      : "memory");
}

// 4-D form: coordinates (c0 innermost .. c3)
__device__ __forceinline__ void tma_load_4d_hint(uint32_t dst, const void* tmap, int c0, int c1,
                                                 int c2, int c3, uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar),
      "l"(policy)
      : "memory");
}

// Same (3-D), with an L2 cache-policy hint (createpolicy result).
__device__ __forceinline__ void tma_load_3d_hint(uint32_t dst, const void* tmap, int c0, int c1,
                                                 int c2, uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(c0), "r"(c1), "r"(c2), "r"(bar), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// ---------------------------------------------------------------------------
// tcgen05: TMEM allocation, MMA, commit, loads/stores, fences
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
// Warpgroup register re-split (all 128 threads of the warpgroup execute it).
template <int N>
__device__ __forceinline__ void setmaxnreg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void setmaxnreg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}

// UMMA shared-memory matrix descriptor, 128-byte swizzle (tcgen05 "version 1"
// layout: start>>4 @0, LBO>>4 @16, SBO>>4 @32, version=1 @46, swizzle mode 2 @61).
__device__ __forceinline__ uint64_t make_desc_sw128(uint32_t saddr, uint32_t lbo_bytes,
                                                    uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;
  d |= 2ull << 61;
  return d;
}

// Instruction descriptor for kind::f16 / kind::f8f6f4 dense MMA with fp32 accumulation.
// fmt: kind::f16 -> 0 f16, 1 bf16; kind::f8f6f4 -> 0 e4m3.  major: 0 K-major, 1 MN-major.
__host__ __device__ constexpr uint32_t make_idesc(int M, int N, int a_fmt, int b_fmt, int a_major,
                                                  int b_major) {
  return (1u << 4) | (uint32_t(a_fmt) << 7) | (uint32_t(b_fmt) << 10) |
         (uint32_t(a_major) << 15) | (uint32_t(b_major) << 16) | (uint32_t(N >> 3) << 17) |
         (uint32_t(M >> 4) << 24);
}

// D[tmem] (+)= A[smem desc] * B[smem desc]
__device__ __forceinline__ void mma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc]
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_f8_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_f8_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 32 lanes x 32 bits, 32 consecutive columns: thread i of the warp gets lane
// (warp's lane base + i), columns [taddr.col, taddr.col + 32).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void reg_fence16(uint32_t (&r)[16]) {
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                 "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                 "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]));
}
// 16 columns variant (used for 8-bit P, which packs 4 values per column).
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
// Make the compiler treat the 32 registers as (re)defined here, so no use of a
// tcgen05.ld result is scheduled above the preceding tcgen05.wait::ld.
__device__ __forceinline__ void reg_fence32(uint32_t (&r)[32]) {
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                 "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                 "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]),
                 "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]),
                 "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]),
                 "+r"(r[30]), "+r"(r[31]));
}

// ---------------------------------------------------------------------------
// packed fp32x2 arithmetic (sm_100: one instruction for two lanes of a 64-bit pair)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t f2pack(float lo, float hi) {
  return uint64_t(__float_as_uint(lo)) | (uint64_t(__float_as_uint(hi)) << 32);
}
__device__ __forceinline__ float f2lo(uint64_t v) { return __uint_as_float(uint32_t(v)); }
__device__ __forceinline__ float f2hi(uint64_t v) { return __uint_as_float(uint32_t(v >> 32)); }
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t fmul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 2^x for two lanes on the FMA/ALU pipes instead of the MUFU unit (Cody-Waite range
// reduction x = n + f, n = round(x), |f| <= 1/2, then a cubic in f).  The cubic is this
// project's own minimax fit of 2^f on [-1/2, 1/2] by the Remez exchange algorithm
// (max relative error 7.5e-5, below the rounding of the bf16/f16/e4m3 P it feeds).
// 2^n is applied by adding n to the exponent field.  x is clamped to >= -126, so
// masked (-inf) scores give a denormal ~0 instead of a NaN.
__device__ __forceinline__ uint64_t exp2_poly_x2(uint64_t x) {
  const float x0 = fmaxf(f2lo(x), -126.0f), x1 = fmaxf(f2hi(x), -126.0f);
  const uint64_t xc = f2pack(x0, x1);
  const uint64_t round_c = f2pack(12582912.0f, 12582912.0f);    // 1.5 * 2^23
  const uint64_t neg_round_c = f2pack(-12582912.0f, -12582912.0f);
  const uint64_t minus1 = f2pack(-1.0f, -1.0f);
  const uint64_t t = fadd2(xc, round_c);        // low mantissa bits of t hold round(x)
  const uint64_t n = fadd2(t, neg_round_c);     // round(x) as a float
  const uint64_t f = ffma2(n, minus1, xc);      // x - round(x), in [-1/2, 1/2]
  uint64_t p = ffma2(f, f2pack(0.0551716685f, 0.0551716685f), f2pack(0.242611125f, 0.242611125f));
  p = ffma2(p, f, f2pack(0.693260968f, 0.693260968f));
  p = ffma2(p, f, f2pack(0.999928057f, 0.999928057f));
  const uint32_t r0 = uint32_t(p) + (uint32_t(t) << 23);
  const uint32_t r1 = uint32_t(p >> 32) + (uint32_t(t >> 32) << 23);
  return uint64_t(r0) | (uint64_t(r1) << 32);
}

// Degree-2 form of the same reduction (own minimax fit of 2^f on [-1/2, 1/2] by the same
// Remez exchange; max relative error 1.7e-3): enough for an e4m3 P, whose rounding step is
// 2^-3 relative, at two FMAs per element pair fewer than the cubic.
__device__ __forceinline__ uint64_t exp2_poly2_x2(uint64_t x) {
  const float x0 = fmaxf(f2lo(x), -126.0f), x1 = fmaxf(f2hi(x), -126.0f);
  const uint64_t xc = f2pack(x0, x1);
  const uint64_t t = fadd2(xc, f2pack(12582912.0f, 12582912.0f));  // 1.5 * 2^23
  const uint64_t n = fadd2(t, f2pack(-12582912.0f, -12582912.0f));
  const uint64_t f = ffma2(n, f2pack(-1.0f, -1.0f), xc);
  uint64_t p = ffma2(f, f2pack(0.238428935f, 0.238428935f), f2pack(0.703447998f, 0.703447998f));
  p = ffma2(p, f, f2pack(1.00044310f, 1.00044310f));
  const uint32_t r0 = uint32_t(p) + (uint32_t(t) << 23);
  const uint32_t r1 = uint32_t(p >> 32) + (uint32_t(t >> 32) << 23);
  return uint64_t(r0) | (uint64_t(r1) << 32);
}

// ---------------------------------------------------------------------------
// packing helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
// four floats -> four e4m3 bytes (satfinite), lowest float in the lowest byte
__device__ __forceinline__ uint32_t pack_e4m3x4(float a, float b, float c, float d) {
  uint16_t lo, hi;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(lo) : "f"(b), "f"(a));
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(hi) : "f"(d), "f"(c));
  return uint32_t(lo) | (uint32_t(hi) << 16);
}
// inverse of pack_e4m3x4 (exact: every e4m3 value is an f16 value)
__device__ __forceinline__ void unpack_e4m3x4(uint32_t w, float& a, float& b, float& c, float& d) {
  uint32_t lo, hi;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(lo) : "h"(uint16_t(w & 0xFFFFu)));
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(hi) : "h"(uint16_t(w >> 16)));
  const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&lo));
  const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&hi));
  a = f0.x; b = f0.y; c = f1.x; d = f1.y;
}

}  // namespace fa4cp
