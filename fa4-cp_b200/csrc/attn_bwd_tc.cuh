// NEXT BACKWARD KERNEL, STAGED: not included by any translation unit of the library and not yet
// run on a GPU (the shipped backward is attn_bwd.cu).  tcgen05 / TMEM attention backward.
// Its offsets, descriptors and TMEM column maps are checked on the CPU by a numpy model of the
// data flow (tests/test_bwd_tc_model.py) and it is compile-checked for sm_100a there too; it
// is wired into fa4cp_attn_bwd only after GPU parity against the oracle.
// One CTA = 128 keys (TMEM lanes) of one kv head of one sequence; walks the GQA group's query
// heads and the 64-row query tiles that see its keys.
//
// TMEM (512 columns): ST [0,64) S^T fp32 (P^T bf16 in [0,32) after softmax) | DPT [64,128)
// dP^T (dS^T bf16 in [64,96)) | DV [128,256) | DK [256,384) | DQT0 [384,448) | DQT1 [448,512)
// (dQ^T = K^T dS^T, lanes = head dim, double-buffered).
//
// MMAs per query tile t (Q/dO buffer b = t & 1):
//   S^T  = K  Q^T  : SS, A = K tile K-major, B = Q tile K-major        (M 128, N 64)
//   dP^T = V  dO^T : SS, A = V tile K-major, B = dO tile K-major       (M 128, N 64)
//   dV  += P^T dO  : TS, A = ST columns (bf16), B = dO tile MN-major   (M 128, N 128)
//   dK  += dS^T Q  : TS, A = DPT columns (bf16), B = Q tile MN-major   (M 128, N 128)
//   dQ^T = K^T dS^T: SS, A = K tile MN-major, B = dS^T smem MN-major   (M 128, N 64)
//
// Warps: 0 TMA producer, 1 MMA issuer, 2 TMEM allocator, 3 idle (warpgroup 0, 56 regs);
// 4-7 softmax (lane = key; P^T, dS^T; dS^T also to smem; final dK/dV epilogue);
// 8-11 dQ epilogue (lane = head-dim element; vector of 64 queries -> red.add to HBM).
#pragma once
#include <atomic>

#include "common.cuh"

namespace fa4cp {
#ifndef FA4CP_BWD_TC_IN_FWD_TU
// compile check on its own; inside the library it is included where g_attn_status lives
__device__ int g_attn_status = 0;
#endif
namespace bwdtc {

constexpr int D = 128;
constexpr int BN = 128;            // keys per CTA
constexpr int BMQ = 64;            // queries per tile
constexpr int THREADS = 384;
constexpr int CHUNK = 64;          // 16-bit elements per 128-byte swizzle row
constexpr int K_CHUNK_BYTES = BN * 128;     // [128 rows x 128 B]
constexpr int Q_CHUNK_BYTES = BMQ * 128;    // [64 rows x 128 B]
constexpr int KV_BYTES = BN * D * 2;        // 32 KB
constexpr int Q_BYTES = BMQ * D * 2;        // 16 KB
constexpr int DS_BYTES = BN * BMQ * 2;      // 16 KB: [128 keys x 64 queries] bf16
constexpr int OFF_K = 0;
constexpr int OFF_V = OFF_K + KV_BYTES;
constexpr int OFF_Q = OFF_V + KV_BYTES;            // 2 buffers
constexpr int OFF_O = OFF_Q + 2 * Q_BYTES;         // 2 buffers (dO)
constexpr int OFF_DS = OFF_O + 2 * Q_BYTES;        // 2 buffers
constexpr int OFF_LD = OFF_DS + 2 * DS_BYTES;      // [2][2][64] floats: LSE, Delta
constexpr int OFF_BAR = OFF_LD + 2 * 2 * BMQ * 4;
// kv_full, q_full[2], q_empty[2], s_full, p_full, ds_free[2], dq_full[2], dq_free[2], kv_done, td
constexpr int NUM_BARS = 1 + 2 + 2 + 1 + 1 + 2 + 2 + 2 + 1 + 1;
constexpr int SMEM_BYTES = OFF_BAR + NUM_BARS * 8 + 16 + 1024;
static_assert(SMEM_BYTES <= 232448, "shared memory budget");
constexpr int TM_ST = 0, TM_DPT = 64, TM_DV = 128, TM_DK = 256, TM_DQT = 384;
constexpr int TM_COLS = 512;
constexpr int REGS_LOW = 56, REGS_HIGH = 224;
static_assert(128 * (REGS_LOW + 2 * REGS_HIGH) <= THREADS * 168, "register re-split");

constexpr int kErrBase = 0x300;

struct Params {
  const float* lse;
  const float* delta;
  float* dq;
  float* dk;
  float* dv;
  const int32_t* cu_q;
  const int32_t* cu_k;
  int Hq, Hkv, group, pattern, causal, in_fmt;
  float scale, scale_log2;
};

struct Geo {
  int qs, ql, ks, kl;
};

__device__ __forceinline__ Geo geometry(const Params& p, int seq) {
  Geo g;
  const int a = p.cu_q[seq], b = p.cu_q[seq + 1];
  if (p.pattern == FA4CP_PATTERN_VARLEN) {
    g.qs = a; g.ql = b - a; g.ks = p.cu_k[seq]; g.kl = p.cu_k[seq + 1] - g.ks;
  } else {
    const int n = b - a, hh = n / 2;
    if (p.pattern == FA4CP_PATTERN_FRONT_KV) {
      g.qs = a; g.ql = n; g.ks = a; g.kl = hh;
    } else {
      g.qs = a + hh; g.ql = n - hh; g.ks = a; g.kl = n;
    }
  }
  return g;
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void named_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}
__device__ __forceinline__ void red_add_f32(float* p, float v) {
  asm volatile("red.global.add.f32 [%0], %1;" ::"l"(p), "f"(v) : "memory");
}

__global__ void __launch_bounds__(THREADS, 1)
    attn_bwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ,
                       const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV,
                       const __grid_constant__ CUtensorMap tmO, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  const uint32_t bar0 = smem_u32(bars);
  auto BAR = [&](int i) -> uint32_t { return bar0 + 8u * uint32_t(i); };
  const uint32_t kv_full = BAR(0);
  auto q_full = [&](int b) { return BAR(1 + b); };
  auto q_empty = [&](int b) { return BAR(3 + b); };
  const uint32_t s_full = BAR(5);
  const uint32_t p_full = BAR(6);
  auto ds_free = [&](int b) { return BAR(7 + b); };
  auto dq_full = [&](int b) { return BAR(9 + b); };
  auto dq_free = [&](int b) { return BAR(11 + b); };
  const uint32_t kv_done = BAR(13);
  const uint32_t td_bar = BAR(14);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + NUM_BARS);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* status = &g_attn_status;

  // work of this CTA (uniform over the CTA)
  const int seq = blockIdx.z, hk = blockIdx.x;
  const Geo geo = geometry(p, seq);
  const int k0 = blockIdx.y * BN;
  int q_first = 0;
  if (p.causal) {
    q_first = k0 - (geo.kl - geo.ql);
    if (q_first < 0) q_first = 0;
    q_first = (q_first / BMQ) * BMQ;
  }
  if (k0 >= geo.kl || geo.ql <= 0 || q_first >= geo.ql) return;
  const int n_qt = (geo.ql - q_first + BMQ - 1) / BMQ;
  const int n_tiles = p.group * n_qt;
  auto tile_q0 = [&](int t) { return q_first + (t % n_qt) * BMQ; };
  auto tile_head = [&](int t) { return hk * p.group + t / n_qt; };

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(q_full(b), 1);
      mbar_init(q_empty(b), 1);
      mbar_init(ds_free(b), 1);
      mbar_init(dq_full(b), 1);
      mbar_init(dq_free(b), 128);
    }
    mbar_init(s_full, 1);
    mbar_init(p_full, 128);
    mbar_init(kv_done, 1);
    mbar_init(td_bar, 1);
    *abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    tma_prefetch_desc(&tmO);
  }
  if (warp == 2) {
    tmem_alloc(smem_u32(tmem_slot), TM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp < 4) {
    setmaxnreg_dec<REGS_LOW>();
    if (warp == 0 && lane == 0) {
      // ------------------------------------------------------------ TMA producer
      mbar_arrive_expect_tx(kv_full, 2 * KV_BYTES);
      for (int c = 0; c < D / CHUNK; ++c) {
        tma_load_3d(smem_u32(smem + OFF_K + c * K_CHUNK_BYTES), &tmK, c * CHUNK, hk, geo.ks + k0,
                    kv_full);
        tma_load_3d(smem_u32(smem + OFF_V + c * K_CHUNK_BYTES), &tmV, c * CHUNK, hk, geo.ks + k0,
                    kv_full);
      }
      for (int t = 0; t < n_tiles; ++t) {
        const int b = t & 1;
        if (t >= 2 && !mbar_wait(q_empty(b), ((t >> 1) - 1) & 1, abort, kErrBase + 1, status)) break;
        mbar_arrive_expect_tx(q_full(b), 2 * Q_BYTES);
        const int row = geo.qs + tile_q0(t), hq = tile_head(t);
        for (int c = 0; c < D / CHUNK; ++c) {
          tma_load_3d(smem_u32(smem + OFF_Q + b * Q_BYTES + c * Q_CHUNK_BYTES), &tmQ, c * CHUNK,
                      hq, row, q_full(b));
          tma_load_3d(smem_u32(smem + OFF_O + b * Q_BYTES + c * Q_CHUNK_BYTES), &tmO, c * CHUNK,
                      hq, row, q_full(b));
        }
      }
      // every copy issued has landed before the role ends
      mbar_wait_drain(kv_full, 0, kErrBase + 2, status);
      for (int b = 0; b < 2 && b < n_tiles; ++b) {
        const int last = ((n_tiles - 1 - b) / 2) * 2 + b;  // last tile that used buffer b
        mbar_wait_drain(q_full(b), (last >> 1) & 1, kErrBase + 2, status);
      }
    } else if (warp == 1 && lane == 0) {
      // ------------------------------------------------------------ MMA issuer
      const int fmt = p.in_fmt;
      const uint32_t id_s = make_idesc(128, BMQ, fmt, fmt, 0, 0);    // S^T, dP^T
      const uint32_t id_dkv = make_idesc(128, D, fmt, fmt, 0, 1);    // dV, dK (A from TMEM)
      const uint32_t id_dq = make_idesc(128, BMQ, fmt, fmt, 1, 1);   // dQ^T: both MN-major
      const uint32_t sK = smem_u32(smem + OFF_K), sV = smem_u32(smem + OFF_V);
      bool ok = mbar_wait(kv_full, 0, abort, kErrBase + 3, status);
      tc_fence_after();
      for (int t = 0; ok && t < n_tiles; ++t) {
        const int b = t & 1;
        const uint32_t sQ = smem_u32(smem + OFF_Q + b * Q_BYTES);
        const uint32_t sO = smem_u32(smem + OFF_O + b * Q_BYTES);
        const uint32_t sDS = smem_u32(smem + OFF_DS + b * DS_BYTES);
        if (!(ok = mbar_wait(q_full(b), (t >> 1) & 1, abort, kErrBase + 4, status))) break;
        tc_fence_after();
        // S^T and dP^T (K-steps over the head dim)
        for (int kk = 0; kk < D / 16; ++kk) {
          const int off = kk * 32;
          const uint32_t ca = (off / 128) * K_CHUNK_BYTES + (off % 128);
          const uint32_t cb = (off / 128) * Q_CHUNK_BYTES + (off % 128);
          mma_f16_ss(tmem + TM_ST, make_desc_sw128(sK + ca, 16, 1024),
                     make_desc_sw128(sQ + cb, 16, 1024), id_s, kk > 0 ? 1u : 0u);
          mma_f16_ss(tmem + TM_DPT, make_desc_sw128(sV + ca, 16, 1024),
                     make_desc_sw128(sO + cb, 16, 1024), id_s, kk > 0 ? 1u : 0u);
        }
        tc_commit(s_full);
        // P^T, dS^T (TMEM) and dS^T (smem) from the softmax warps
        if (!(ok = mbar_wait(p_full, t & 1, abort, kErrBase + 5, status))) break;
        tc_fence_after();
        for (int kk = 0; kk < BMQ / 16; ++kk) {  // K-steps over the tile's queries
          const uint64_t bo = make_desc_sw128(sO + kk * 16 * 128, Q_CHUNK_BYTES, 1024);
          const uint64_t bq = make_desc_sw128(sQ + kk * 16 * 128, Q_CHUNK_BYTES, 1024);
          const uint32_t acc = (t > 0 || kk > 0) ? 1u : 0u;
          mma_f16_ts(tmem + TM_DV, tmem + TM_ST + kk * 8, bo, id_dkv, acc);
          mma_f16_ts(tmem + TM_DK, tmem + TM_DPT + kk * 8, bq, id_dkv, acc);
        }
        tc_commit(q_empty(b));  // the Q / dO tile's last readers
        // dQ^T = K^T dS^T into buffer b (its previous contents read by the dQ epilogue)
        if (t >= 2 && !(ok = mbar_wait(dq_free(b), ((t >> 1) - 1) & 1, abort, kErrBase + 6, status)))
          break;
        tc_fence_after();
        for (int kk = 0; kk < BN / 16; ++kk) {  // K-steps over the keys
          const uint64_t ak = make_desc_sw128(sK + kk * 16 * 128, K_CHUNK_BYTES, 1024);
          const uint64_t bs = make_desc_sw128(sDS + kk * 16 * 128, DS_BYTES, 1024);
          mma_f16_ss(tmem + TM_DQT + b * BMQ, ak, bs, id_dq, kk > 0 ? 1u : 0u);
        }
        tc_commit(dq_full(b));
        tc_commit(ds_free(b));
      }
      tc_commit(kv_done);
      tc_commit(td_bar);
      mbar_wait_drain(td_bar, 0, kErrBase + 7, status);
    }
  } else if (warp < 8) {
    setmaxnreg_inc<REGS_HIGH>();
    // ------------------------------------------------------------ softmax (lane = key)
    const int wq = warp & 3;
    const int r = wq * 32 + lane;          // key row in the tile / TMEM lane
    const int key = k0 + r;
    const uint32_t t_lane = tmem + (uint32_t(wq * 32) << 16);
    float* ld_s = reinterpret_cast<float*>(smem + OFF_LD);
    uint8_t* ds_s = smem + OFF_DS;
    const int shift = geo.kl - geo.ql;
    bool aborted = false;
    // Every softmax warp runs every trip of this loop and reaches every named_sync(1, 128)
    // (which needs all four warps) even after a bounded wait of its own gave up: a give-up
    // only skips the waits and the work of the later trips.  Leaving the loop early would
    // strand the other warps at the named barrier.
    for (int t = 0; t < n_tiles; ++t) {
      const int b = t & 1;
      const int q0 = tile_q0(t), hq = tile_head(t);
      float* lse_t = ld_s + b * 2 * BMQ;
      float* del_t = lse_t + BMQ;
      // this tile's LSE (natural log -> log2, +inf where no key / past the end) and Delta
      if (!aborted) {
        const int i = r & (BMQ - 1);
        const bool ok_row = q0 + i < geo.ql;
        const int64_t idx = (int64_t(geo.qs) + q0 + i) * p.Hq + hq;
        if (r < BMQ) {
          float l = ok_row ? p.lse[idx] : -__builtin_huge_valf();
          lse_t[i] = (l == -__builtin_huge_valf()) ? __builtin_huge_valf() : l * kLog2e;
        } else {
          del_t[i] = ok_row ? p.delta[idx] : 0.f;
        }
      }
      named_sync(1, 128);
      if (aborted) continue;
      bool ok = mbar_wait(s_full, t & 1, abort, kErrBase + 8, status);
      if (!__all_sync(0xffffffffu, ok)) { aborted = true; continue; }
      tc_fence_after();
      uint32_t sv[2][32], dv[2][32];
      tmem_ld32(t_lane + TM_ST, sv[0]);
      tmem_ld32(t_lane + TM_ST + 32, sv[1]);
      tmem_ld32(t_lane + TM_DPT, dv[0]);
      tmem_ld32(t_lane + TM_DPT + 32, dv[1]);
      tmem_wait_ld();
      reg_fence32(sv[0]); reg_fence32(sv[1]); reg_fence32(dv[0]); reg_fence32(dv[1]);
      uint32_t pw[32], dw[32];
#pragma unroll
      for (int c = 0; c < 2; ++c)
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          float pr[2], ds[2];
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int qi = c * 32 + e + u;
            const bool vis = key < geo.kl && (!p.causal || key <= q0 + qi + shift);
            const float x = __uint_as_float(sv[c][e + u]) * p.scale_log2 - lse_t[qi];
            pr[u] = vis ? ex2_approx(x) : 0.f;
            ds[u] = pr[u] * (__uint_as_float(dv[c][e + u]) - del_t[qi]);
          }
          pw[(c * 32 + e) / 2] = p.in_fmt ? pack_bf16x2(pr[0], pr[1]) : pack_f16x2(pr[0], pr[1]);
          dw[(c * 32 + e) / 2] = p.in_fmt ? pack_bf16x2(ds[0], ds[1]) : pack_f16x2(ds[0], ds[1]);
        }
      // dS^T row r into the MN-major smem tile of buffer b (128-byte rows, 16-byte chunks
      // XOR-swizzled by r % 8, as a 128-byte-swizzled TMA copy would place them)
      if (t >= 2) {
        ok = mbar_wait(ds_free(b), ((t >> 1) - 1) & 1, abort, kErrBase + 9, status);
        if (!__all_sync(0xffffffffu, ok)) { aborted = true; continue; }
      }
      uint8_t* row = ds_s + b * DS_BYTES + r * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c)
        *reinterpret_cast<uint4*>(row + ((c ^ (r & 7)) * 16)) =
            make_uint4(dw[4 * c], dw[4 * c + 1], dw[4 * c + 2], dw[4 * c + 3]);
      fence_proxy_async_smem();
      tmem_st32(t_lane + TM_ST, pw);
      tmem_st32(t_lane + TM_DPT, dw);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(p_full);
    }
    // dK / dV of this key row into the fp32 accumulators
    if (!aborted) {
      bool ok = mbar_wait(kv_done, 0, abort, kErrBase + 10, status);
      if (__all_sync(0xffffffffu, ok) && key < geo.kl) {
        tc_fence_after();
        float* dkr = p.dk + ((int64_t(geo.ks) + key) * p.Hkv + hk) * int64_t(D);
        float* dvr = p.dv + ((int64_t(geo.ks) + key) * p.Hkv + hk) * int64_t(D);
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t a[32], v[32];
          tmem_ld32(t_lane + TM_DK + c * 32, a);
          tmem_ld32(t_lane + TM_DV + c * 32, v);
          tmem_wait_ld();
          reg_fence32(a);
          reg_fence32(v);
#pragma unroll
          for (int e = 0; e < 32; e += 4) {
            float4* pk = reinterpret_cast<float4*>(dkr + c * 32 + e);
            float4* pv = reinterpret_cast<float4*>(dvr + c * 32 + e);
            float4 x = *pk, y = *pv;
            x.x += __uint_as_float(a[e]) * p.scale; x.y += __uint_as_float(a[e + 1]) * p.scale;
            x.z += __uint_as_float(a[e + 2]) * p.scale; x.w += __uint_as_float(a[e + 3]) * p.scale;
            y.x += __uint_as_float(v[e]); y.y += __uint_as_float(v[e + 1]);
            y.z += __uint_as_float(v[e + 2]); y.w += __uint_as_float(v[e + 3]);
            *pk = x;
            *pv = y;
          }
        }
      }
    }
  } else {
    setmaxnreg_inc<REGS_HIGH>();
    // ------------------------------------------------------------ dQ epilogue (lane = d)
    const int wq = warp & 3;
    const int d = wq * 32 + lane;
    const uint32_t t_lane = tmem + (uint32_t(wq * 32) << 16);
    for (int t = 0; t < n_tiles; ++t) {
      const int b = t & 1;
      bool ok = mbar_wait(dq_full(b), (t >> 1) & 1, abort, kErrBase + 11, status);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      uint32_t v[2][32];
      tmem_ld32(t_lane + TM_DQT + b * BMQ, v[0]);
      tmem_ld32(t_lane + TM_DQT + b * BMQ + 32, v[1]);
      tmem_wait_ld();
      reg_fence32(v[0]);
      reg_fence32(v[1]);
      tc_fence_before();
      mbar_arrive(dq_free(b));
      const int q0 = tile_q0(t), hq = tile_head(t);
      const int nrow = geo.ql - q0 < BMQ ? geo.ql - q0 : BMQ;
      float* base = p.dq + ((int64_t(geo.qs) + q0) * p.Hq + hq) * int64_t(D) + d;
      const int64_t stride = int64_t(p.Hq) * D;
#pragma unroll
      for (int c = 0; c < 2; ++c)
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int qi = c * 32 + e;
          if (qi < nrow) red_add_f32(base + qi * stride, __uint_as_float(v[c][e]) * p.scale);
        }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 2) tmem_dealloc(tmem, TM_COLS);
}

}  // namespace bwdtc
}  // namespace fa4cp

// ---------------------------------------------------------------------------------------
// host launcher (draft): tensor maps as the forward's make_map (3-D [rows, heads, D], 128-byte
// swizzled boxes of 64 elements x 1 head x box_rows)
// ---------------------------------------------------------------------------------------
namespace fa4cp {
namespace bwdtc {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static int map3(CUtensorMap* m, const void* base, int64_t rows, int heads, int box_rows) {
  static EncodeTiledFn enc = nullptr;
  if (enc == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess && q == cudaDriverEntryPointSuccess)
      enc = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  if (enc == nullptr) return FA4CP_ERR_CUDA;
  const cuuint64_t dims[3] = {cuuint64_t(D), cuuint64_t(heads), cuuint64_t(rows)};
  const cuuint64_t strides[2] = {cuuint64_t(D) * 2, cuuint64_t(heads) * D * 2};
  const cuuint32_t box[3] = {64, 1, cuuint32_t(box_rows)};
  const cuuint32_t es[3] = {1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<void*>(base), dims, strides, box,
             es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS
             ? FA4CP_OK : FA4CP_ERR_CUDA;
}

// same arguments as fa4cp_attn_bwd (head_dim 128 only)
int launch(const void* q, const void* k, const void* v, const void* dout, const Params& p,
           int64_t total_q, int64_t total_k, int nseq, int max_seqlen_k, cudaStream_t st) {
  static std::atomic<uint64_t> optin{0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return FA4CP_ERR_CUDA;
  const uint64_t bit = dev < 64 ? (uint64_t(1) << dev) : 0;
  if (bit == 0 || !(optin.load() & bit)) {
    if (cudaFuncSetAttribute(attn_bwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             SMEM_BYTES) != cudaSuccess)
      return FA4CP_ERR_CUDA;
    optin.fetch_or(bit);
  }
  CUtensorMap mq, mk, mv, mo;
  int rc;
  if ((rc = map3(&mq, q, total_q, p.Hq, BMQ))) return rc;
  if ((rc = map3(&mo, dout, total_q, p.Hq, BMQ))) return rc;
  if ((rc = map3(&mk, k, total_k, p.Hkv, BN))) return rc;
  if ((rc = map3(&mv, v, total_k, p.Hkv, BN))) return rc;
  const int tiles = (max_seqlen_k + BN - 1) / BN;
  if (tiles <= 0) return FA4CP_OK;
  dim3 grid(unsigned(p.Hkv), unsigned(tiles), unsigned(nseq));
  attn_bwd_tc_kernel<<<grid, THREADS, SMEM_BYTES, st>>>(mq, mk, mv, mo, p);
  return cudaGetLastError() == cudaSuccess ? FA4CP_OK : FA4CP_ERR_CUDA;
}

}  // namespace bwdtc
}  // namespace fa4cp
