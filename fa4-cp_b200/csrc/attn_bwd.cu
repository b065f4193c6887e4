// Attention backward for the zig-zag ring: dQ, dK, dV of one ring step (any of the three
// step patterns, or plain varlen attention), f16 / bf16 inputs, fp32 accumulation.
//
// The reference is forward-only (its README's "forward-only (inference). No backward",
// README.md:142); this is the gradient of its forward (tests/test_algorithm_cpu.py:36-48,
// the per-step row selections of fa4_ring/ring_attention.py:109-166).  Per head, with the
// FINAL natural-log LSE of every query row (so that the partial gradients of the ring steps
// add up):
//   P = exp(scale * Q K^T - LSE),  Delta_i = sum_d dO_id * O_id
//   dV = P^T dO,  dS = P * (dO V^T - Delta),  dQ = scale * dS K,  dK = scale * dS^T Q
//
// Kernel layout (one CTA = 128 keys of one kv head of one sequence, 8 warps x 16 keys):
//   * the CTA's K and V tiles stay in shared memory for its whole life;
//   * it walks the query heads of its GQA group and, per head, the 32-row query tiles that can
//     see its keys (causal: from the first visible tile on); Q, dO, LSE and Delta of the next
//     tile load with cp.async (double-buffered) while the current one computes;
//   * each warp computes S^T and dP^T for its 16 keys (mma.sync m16n8k16, fp32 accumulators,
//     operand fragments by ldmatrix, transposed where the operand is stored k-major), forms
//     P^T and dS^T in registers, and accumulates dV and dK for its keys in registers;
//   * dS^T goes through shared memory so that all 8 warps compute the tile's dQ = dS K, which is
//     added to an fp32 dQ accumulator in HBM with vector atomics (many key tiles add into one
//     query row);
//   * at the end, dK and dV are added to fp32 accumulators (one CTA owns each key row within a
//     launch, so a plain read-add-write).
// The accumulators are fp32 so that the ring can add the contributions of all its steps
// before one rounding to the input dtype.
#include <atomic>
#include <type_traits>

#include "common.cuh"

namespace fa4cp {
namespace {

#ifndef FA4CP_BWD_BN
#define FA4CP_BWD_BN 128
#endif
constexpr int kBwdBN = FA4CP_BWD_BN;     // keys per CTA (64 or 128)
constexpr int kBwdBM = 32;               // query rows per inner tile
constexpr int kBwdWarps = kBwdBN / 16;   // one warp per 16 keys
constexpr int kBwdThreads = kBwdWarps * 32;
constexpr int kBwdMinBlocks = kBwdBN == 64 ? 2 : 1;  // CTAs per SM the registers allow
static_assert(kBwdBN == 64 || kBwdBN == 128, "64 or 128 keys per CTA");

template <typename T> struct Mma16;
template <> struct Mma16<__nv_bfloat16> {
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) { return pack_bf16x2(lo, hi); }
  static __device__ __forceinline__ void mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                             uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
};
template <> struct Mma16<__half> {
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) { return pack_f16x2(lo, hi); }
  static __device__ __forceinline__ void mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                             uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
};

// two consecutive 16-bit elements (the lower address in the low half)
__device__ __forceinline__ uint32_t ld_pair(const uint16_t* p) {
  return *reinterpret_cast<const uint32_t*>(p);
}

// four 8x8 16-bit matrices from shared memory; lanes 8m..8m+7 give the row addresses of
// matrix m.  Plain: thread t receives row t/4, columns 2(t%4), 2(t%4)+1 of each matrix;
// .trans: rows 2(t%4), 2(t%4)+1 of column t/4.
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// asynchronous global -> shared copies; src_bytes 0 reads nothing and zero-fills
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
               "r"(src_bytes));
}
__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src, int src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src),
               "r"(src_bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N));
}

struct BwdParams {
  const void* q;
  const void* k;
  const void* v;
  const void* dout;
  const float* lse;
  const float* delta;
  float* dq;
  float* dk;
  float* dv;
  const int32_t* cu_q;
  const int32_t* cu_k;
  int Hq, Hkv, group;
  int pattern;
  int causal;
  float scale;
  float scale_log2;
};

struct BwdGeo {
  int qs, ql, ks, kl;
};

// the rows one ring step covers in sequence `seq` (the forward's seq_geometry)
__device__ __forceinline__ BwdGeo bwd_geometry(const BwdParams& p, int seq) {
  BwdGeo g;
  const int a = p.cu_q[seq], b = p.cu_q[seq + 1];
  if (p.pattern == FA4CP_PATTERN_VARLEN) {
    g.qs = a;
    g.ql = b - a;
    g.ks = p.cu_k[seq];
    g.kl = p.cu_k[seq + 1] - g.ks;
  } else {
    const int n = b - a, hh = n / 2;
    if (p.pattern == FA4CP_PATTERN_FRONT_KV) {
      g.qs = a; g.ql = n; g.ks = a; g.kl = hh;
    } else {  // FA4CP_PATTERN_BACK_Q
      g.qs = a + hh; g.ql = n - hh; g.ks = a; g.kl = n;
    }
  }
  return g;
}

// shared memory (16-bit elements unless noted): K and V tiles for the CTA's life; Q and dO
// tiles double-buffered (the next query tile loads while this one computes); the dS^T tile;
// then LSE and Delta rows (float, double-buffered)
template <int D>
struct BwdSmem {
  static constexpr int LDK = D + 8;            // row pitch of K / V / Q / dO tiles
  static constexpr int LDS = kBwdBM + 8;       // row pitch of the dS^T tile
  static constexpr int TILE = kBwdBM * LDK;    // one Q or dO tile
  static constexpr int K_OFF = 0;
  static constexpr int V_OFF = K_OFF + kBwdBN * LDK;
  static constexpr int Q_OFF = V_OFF + kBwdBN * LDK;
  static constexpr int O_OFF = Q_OFF + 2 * TILE;
  static constexpr int S_OFF = O_OFF + 2 * TILE;
  static constexpr int HALVES = S_OFF + kBwdBN * LDS;
  static constexpr int BYTES = HALVES * 2 + 2 * 2 * kBwdBM * 4;
  static_assert((LDK * 2) % 16 == 0 && (LDS * 2) % 16 == 0 && (HALVES * 2) % 16 == 0,
                "16-byte rows");
};

// rows [row0, row0 + nrows) of a [rows, heads, D] tensor, head `h`, into a pitch-LDK tile
// with cp.async; rows at or past `valid` are zero-filled (no global read)
template <int D, int NROWS>
__device__ __forceinline__ void stage_rows_async(uint16_t* dst, const uint16_t* src,
                                                 int64_t row0, int valid, int heads, int h) {
  constexpr int CPR = D / 8;  // 16-byte chunks per row
  constexpr int LDK = BwdSmem<D>::LDK;
  for (int c = threadIdx.x; c < NROWS * CPR; c += kBwdThreads) {
    const int r = c / CPR, col = (c % CPR) * 8;
    const bool ok = r < valid;
    const uint16_t* g = ok ? src + ((row0 + r) * heads + h) * int64_t(D) + col : src;
    cp_async16(smem_u32(dst + r * LDK + col), g, ok ? 16 : 0);
  }
}

template <typename T, int D>
__global__ void __launch_bounds__(kBwdThreads, kBwdMinBlocks) attn_bwd_kernel(const BwdParams p) {
  using SM = BwdSmem<D>;
  constexpr int LDK = SM::LDK, LDS = SM::LDS;
  constexpr int NT_D = D / 8;          // n-tiles over the head dim
  constexpr int NT_Q = kBwdBM / 8;     // n-tiles over a query tile
  constexpr int NQ = NT_D / (kBwdWarps / 2);  // dQ n-tiles per warp (2 m-tiles x warps/2 columns)
  static_assert(NT_Q % 2 == 0 && NQ % 2 == 0, "n-tiles are loaded in pairs");
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint16_t* sh = reinterpret_cast<uint16_t*>(smem_raw);
  uint16_t* sK = sh + SM::K_OFF;
  uint16_t* sV = sh + SM::V_OFF;
  uint16_t* sQ = sh + SM::Q_OFF;
  uint16_t* sO = sh + SM::O_OFF;
  uint16_t* sS = sh + SM::S_OFF;
  float* sL = reinterpret_cast<float*>(sh + SM::HALVES);  // [2][BM] raw LSE
  float* sD = sL + 2 * kBwdBM;                             // [2][BM] Delta

  // grid (kv head, key tile, sequence): the heads' tiles of one key range are adjacent in
  // launch order, so the heaviest (earliest, under a causal mask) key tiles of every head
  // start first and the light ones fill the tail
  const int seq = blockIdx.z, hk = blockIdx.x;
  const BwdGeo geo = bwd_geometry(p, seq);
  const int k0 = blockIdx.y * kBwdBN;
  if (k0 >= geo.kl || geo.ql <= 0) return;  // uniform over the CTA
  int q_first = 0;
  if (p.causal) {  // key j is visible to query i iff j <= i + (kl - ql)
    q_first = k0 - (geo.kl - geo.ql);
    if (q_first < 0) q_first = 0;
    q_first = (q_first / kBwdBM) * kBwdBM;
  }
  if (q_first >= geo.ql) return;
  const int n_qt = (geo.ql - q_first + kBwdBM - 1) / kBwdBM;  // query tiles per head
  const int n_tiles = p.group * n_qt;                         // over the group's heads

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tq = lane & 3;
  const int lm = lane >> 3, lr = lane & 7;  // ldmatrix: matrix and row this lane addresses
  const uint16_t* gq = static_cast<const uint16_t*>(p.q);
  const uint16_t* gk = static_cast<const uint16_t*>(p.k);
  const uint16_t* gv = static_cast<const uint16_t*>(p.v);
  const uint16_t* gdo = static_cast<const uint16_t*>(p.dout);

  // K / V (in the first cp.async group, with query tile 0)
  const int kvalid = geo.kl - k0 < kBwdBN ? geo.kl - k0 : kBwdBN;
  stage_rows_async<D, kBwdBN>(sK, gk, int64_t(geo.ks) + k0, kvalid, p.Hkv, hk);
  stage_rows_async<D, kBwdBN>(sV, gv, int64_t(geo.ks) + k0, kvalid, p.Hkv, hk);

  auto stage_tile = [&](int t, int buf) {
    const int hq = hk * p.group + t / n_qt;
    const int q0 = q_first + (t % n_qt) * kBwdBM;
    const int qvalid = geo.ql - q0 < kBwdBM ? geo.ql - q0 : kBwdBM;
    stage_rows_async<D, kBwdBM>(sQ + buf * SM::TILE, gq, int64_t(geo.qs) + q0, qvalid, p.Hq, hq);
    stage_rows_async<D, kBwdBM>(sO + buf * SM::TILE, gdo, int64_t(geo.qs) + q0, qvalid, p.Hq, hq);
    if (threadIdx.x < kBwdBM) {
      const int r = threadIdx.x;
      const bool ok = r < qvalid;
      const int64_t idx = ok ? (int64_t(geo.qs) + q0 + r) * p.Hq + hq : 0;
      cp_async4(smem_u32(sL + buf * kBwdBM + r), p.lse + idx, ok ? 4 : 0);
      cp_async4(smem_u32(sD + buf * kBwdBM + r), p.delta + idx, ok ? 4 : 0);
    }
    cp_async_commit();
  };

  float dk[NT_D][4], dv[NT_D][4];
#pragma unroll
  for (int n = 0; n < NT_D; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) dk[n][e] = dv[n][e] = 0.f;

  const int krow = warp * 16 + g;     // this thread's first key row in the tile (then + 8)
  const int key0 = k0 + krow;         // its position in the sequence's key range
  const int shift = geo.kl - geo.ql;  // causal alignment (bottom-right)
  const uint32_t sK_a = smem_u32(sK), sV_a = smem_u32(sV), sS_a = smem_u32(sS);
  // byte offsets of this lane's ldmatrix row address within a tile
  //   A (16 K/V rows of the warp x 16 columns): matrices (rows +0/+8) x (columns +0/+8)
  const uint32_t a_off = uint32_t(((warp * 16 + (lm & 1) * 8 + lr) * LDK + (lm >> 1) * 8) * 2);
  //   B from row-major [n][k] (Q, dO as the n side): n-tile pair x (k +0/+8)
  const uint32_t b_off = uint32_t((((lm >> 1) * 8 + lr) * LDK + (lm & 1) * 8) * 2);
  //   B from row-major [k][n] (dO, Q, K as the k side), transposed: (k +0/+8) x n-tile pair
  const uint32_t bt_off = uint32_t((((lm & 1) * 8 + lr) * LDK + (lm >> 1) * 8) * 2);

  stage_tile(0, 0);
  for (int t = 0; t < n_tiles; ++t) {
    const int buf = t & 1;
    if (t + 1 < n_tiles) {
      stage_tile(t + 1, buf ^ 1);  // its last readers (tile t-1) passed tile t-1's dS barrier
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();  // tile t (and K / V) visible to every thread
    const int hq = hk * p.group + t / n_qt;
    const int q0 = q_first + (t % n_qt) * kBwdBM;
    const int qvalid = geo.ql - q0 < kBwdBM ? geo.ql - q0 : kBwdBM;
    const uint32_t sQ_a = smem_u32(sQ + buf * SM::TILE), sO_a = smem_u32(sO + buf * SM::TILE);
    const float* lse_t = sL + buf * kBwdBM;
    const float* del_t = sD + buf * kBwdBM;

    // S^T = K Q^T and dP^T = V dO^T for this warp's 16 keys x 32 queries
    float s[NT_Q][4], dp[NT_Q][4];
#pragma unroll
    for (int n = 0; n < NT_Q; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) s[n][e] = dp[n][e] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t ak[4], av[4];
      ldsm_x4(ak, sK_a + a_off + kk * 32);
      ldsm_x4(av, sV_a + a_off + kk * 32);
#pragma unroll
      for (int np = 0; np < NT_Q / 2; ++np) {
        const uint32_t off = b_off + uint32_t((np * 16 * LDK + kk * 16) * 2);
        uint32_t bq[4], bo[4];
        ldsm_x4(bq, sQ_a + off);
        ldsm_x4(bo, sO_a + off);
        Mma16<T>::mma(s[2 * np], ak, bq[0], bq[1]);
        Mma16<T>::mma(s[2 * np + 1], ak, bq[2], bq[3]);
        Mma16<T>::mma(dp[2 * np], av, bo[0], bo[1]);
        Mma16<T>::mma(dp[2 * np + 1], av, bo[2], bo[3]);
      }
    }

    // P^T and dS^T (element e: key row krow + 8*(e>>1), query column n*8 + 2*tq + (e&1))
#pragma unroll
    for (int n = 0; n < NT_Q; ++n) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int qi = n * 8 + 2 * tq + (e & 1);
        const int key = key0 + ((e & 2) ? 8 : 0);
        const float l = lse_t[qi];
        // a row that sees no key (LSE -inf) or lies past the tile's rows contributes nothing
        const bool vis = qi < qvalid && l != -__builtin_huge_valf() && key < geo.kl &&
                         (!p.causal || key <= q0 + qi + shift);
        const float pr = vis ? ex2_approx(s[n][e] * p.scale_log2 - l * kLog2e) : 0.f;
        s[n][e] = pr;
        dp[n][e] = pr * (dp[n][e] - del_t[qi]);
      }
    }

    // dV += P^T dO and dK += dS^T Q (k = the 32 queries of the tile)
#pragma unroll
    for (int kk = 0; kk < kBwdBM / 16; ++kk) {
      const uint32_t ap[4] = {Mma16<T>::pack(s[2 * kk][0], s[2 * kk][1]),
                              Mma16<T>::pack(s[2 * kk][2], s[2 * kk][3]),
                              Mma16<T>::pack(s[2 * kk + 1][0], s[2 * kk + 1][1]),
                              Mma16<T>::pack(s[2 * kk + 1][2], s[2 * kk + 1][3])};
      const uint32_t ad[4] = {Mma16<T>::pack(dp[2 * kk][0], dp[2 * kk][1]),
                              Mma16<T>::pack(dp[2 * kk][2], dp[2 * kk][3]),
                              Mma16<T>::pack(dp[2 * kk + 1][0], dp[2 * kk + 1][1]),
                              Mma16<T>::pack(dp[2 * kk + 1][2], dp[2 * kk + 1][3])};
#pragma unroll
      for (int jp = 0; jp < NT_D / 2; ++jp) {
        const uint32_t off = bt_off + uint32_t((kk * 16 * LDK + jp * 16) * 2);
        uint32_t bo[4], bq[4];
        ldsm_x4_t(bo, sO_a + off);
        ldsm_x4_t(bq, sQ_a + off);
        Mma16<T>::mma(dv[2 * jp], ap, bo[0], bo[1]);
        Mma16<T>::mma(dv[2 * jp + 1], ap, bo[2], bo[3]);
        Mma16<T>::mma(dk[2 * jp], ad, bq[0], bq[1]);
        Mma16<T>::mma(dk[2 * jp + 1], ad, bq[2], bq[3]);
      }
    }

    // dS^T to shared memory, [key][query]
#pragma unroll
    for (int n = 0; n < NT_Q; ++n) {
      *reinterpret_cast<uint32_t*>(sS + krow * LDS + n * 8 + 2 * tq) =
          Mma16<T>::pack(dp[n][0], dp[n][1]);
      *reinterpret_cast<uint32_t*>(sS + (krow + 8) * LDS + n * 8 + 2 * tq) =
          Mma16<T>::pack(dp[n][2], dp[n][3]);
    }
    __syncthreads();

    // dQ (32 x D) = dS (32 x BN keys) K (BN x D): warp -> m-tile (warp & 1), NQ n-tiles
    {
      const int mt = warp & 1, nb = (warp >> 1) * NQ;
      //   A = dS from the [key][query] tile, transposed: (keys +0/+8) x (queries +0/+8)
      const uint32_t as_off = uint32_t((((lm >> 1) * 8 + lr) * LDS + mt * 16 + (lm & 1) * 8) * 2);
      float dq[NQ][4];
#pragma unroll
      for (int j = 0; j < NQ; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) dq[j][e] = 0.f;
#pragma unroll
      for (int kk = 0; kk < kBwdBN / 16; ++kk) {
        uint32_t a[4];
        ldsm_x4_t(a, sS_a + as_off + uint32_t(kk * 16 * LDS * 2));
#pragma unroll
        for (int jp = 0; jp < NQ / 2; ++jp) {
          uint32_t bk[4];
          ldsm_x4_t(bk, sK_a + bt_off + uint32_t((kk * 16 * LDK + (nb + 2 * jp) * 8) * 2));
          Mma16<T>::mma(dq[2 * jp], a, bk[0], bk[1]);
          Mma16<T>::mma(dq[2 * jp + 1], a, bk[2], bk[3]);
        }
      }
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int qi = mt * 16 + g + 8 * half;
        if (qi < qvalid) {
          float* row = p.dq + ((int64_t(geo.qs) + q0 + qi) * p.Hq + hq) * int64_t(D);
#pragma unroll
          for (int j = 0; j < NQ; ++j) {
            float2* dst = reinterpret_cast<float2*>(row + (nb + j) * 8 + 2 * tq);
            atomicAdd(dst, make_float2(dq[j][2 * half] * p.scale, dq[j][2 * half + 1] * p.scale));
          }
        }
      }
    }
    // no barrier here: the next prefetch into buffer `buf` starts after the barrier above,
    // which every thread reaches after its last read of `buf` (and sL / sD[buf]); the next
    // write of sS comes after the next tile's first barrier, which every thread reaches
    // after this dQ pass
  }

  // dK, dV of this thread's two key rows into the fp32 accumulators
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int key = key0 + 8 * half;
    if (key < geo.kl) {
      const int64_t off = ((int64_t(geo.ks) + key) * p.Hkv + hk) * int64_t(D) + 2 * tq;
#pragma unroll
      for (int n = 0; n < NT_D; ++n) {
        float2* pk = reinterpret_cast<float2*>(p.dk + off + n * 8);
        float2* pv = reinterpret_cast<float2*>(p.dv + off + n * 8);
        float2 a = *pk, b = *pv;
        a.x += dk[n][2 * half] * p.scale;
        a.y += dk[n][2 * half + 1] * p.scale;
        b.x += dv[n][2 * half];
        b.y += dv[n][2 * half + 1];
        *pk = a;
        *pv = b;
      }
    }
  }
}

// Delta[row, head] = sum_d dO * O, one warp per (row, head)
template <typename T>
__global__ void __launch_bounds__(256) bwd_delta_kernel(const uint16_t* __restrict__ out,
                                                        const uint16_t* __restrict__ dout,
                                                        float* __restrict__ delta, int64_t n_rh,
                                                        int D) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = int64_t(gridDim.x) * (blockDim.x >> 5);
  for (int64_t w = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; w < n_rh; w += warps) {
    const uint16_t* o = out + w * D;
    const uint16_t* d = dout + w * D;
    float acc = 0.f;
    for (int c = lane * 2; c < D; c += 64) {
      const uint32_t ov = ld_pair(o + c), dv = ld_pair(d + c);
      float o0, o1, d0, d1;
      if constexpr (sizeof(T) == 2 && std::is_same<T, __nv_bfloat16>::value) {
        o0 = __uint_as_float(ov << 16); o1 = __uint_as_float(ov & 0xFFFF0000u);
        d0 = __uint_as_float(dv << 16); d1 = __uint_as_float(dv & 0xFFFF0000u);
      } else {
        const float2 of = __half22float2(*reinterpret_cast<const __half2*>(&ov));
        const float2 df = __half22float2(*reinterpret_cast<const __half2*>(&dv));
        o0 = of.x; o1 = of.y; d0 = df.x; d1 = df.y;
      }
      acc = fmaf(o0, d0, fmaf(o1, d1, acc));
    }
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, m);
    if (lane == 0) delta[w] = acc;
  }
}

// dst (f16 | bf16 | f32) = src (f32), four elements per thread step
template <typename T>
__global__ void __launch_bounds__(256) convert_f32_kernel(const float* __restrict__ src,
                                                          T* __restrict__ dst, int64_t n) {
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    if constexpr (std::is_same<T, float>::value) {
      dst[i] = src[i];
    } else if constexpr (std::is_same<T, __nv_bfloat16>::value) {
      dst[i] = __float2bfloat16_rn(src[i]);
    } else {
      dst[i] = __float2half_rn(src[i]);
    }
  }
}

__global__ void __launch_bounds__(256) add_f32_kernel(float4* __restrict__ dst,
                                                      const float4* __restrict__ src, int64_t n4) {
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n4; i += stride) {
    float4 a = dst[i];
    const float4 b = src[i];
    a.x += b.x; a.y += b.y; a.z += b.z; a.w += b.w;
    dst[i] = a;
  }
}

unsigned elementwise_grid(int64_t n) {
  static int sms = 0;
  if (sms == 0) {
    int dev = 0, v = 0;
    if (cudaGetDevice(&dev) == cudaSuccess &&
        cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && v > 0)
      sms = v;
    else
      sms = 148;
  }
  const int64_t want = (n + 255) / 256;
  const int64_t cap = int64_t(sms) * 8;
  return unsigned(want < 1 ? 1 : (want < cap ? want : cap));
}

template <typename T, int D>
int launch_bwd(const BwdParams& p, int nseq, int max_seqlen_k, cudaStream_t st) {
  static std::atomic<uint64_t> optin{0};
  int dev = 0;
  FA4CP_CHECK_CUDA(cudaGetDevice(&dev));
  const uint64_t bit = dev < 64 ? (uint64_t(1) << dev) : 0;
  if (bit == 0 || !(optin.load() & bit)) {
    FA4CP_CHECK_CUDA(cudaFuncSetAttribute(attn_bwd_kernel<T, D>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          BwdSmem<D>::BYTES));
    optin.fetch_or(bit);
  }
  const int tiles = (max_seqlen_k + kBwdBN - 1) / kBwdBN;
  if (tiles <= 0) return FA4CP_OK;
  FA4CP_CHECK_ARG(tiles <= 65535, "max_seqlen_k too large");
  dim3 grid(unsigned(p.Hkv), unsigned(tiles), unsigned(nseq));
  attn_bwd_kernel<T, D><<<grid, kBwdThreads, BwdSmem<D>::BYTES, st>>>(p);
  return check_launch("attn_bwd");
}

bool al16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

}  // namespace
}  // namespace fa4cp

using namespace fa4cp;

extern "C" int fa4cp_attn_bwd_preprocess(const void* out, const void* dout, float* delta,
                                         int64_t total_q, int32_t num_heads_q, int32_t head_dim,
                                         int32_t dtype, void* stream) {
  FA4CP_CHECK_ARG(total_q >= 0 && num_heads_q > 0, "bad sizes");
  FA4CP_CHECK_ARG(head_dim > 0 && head_dim % 2 == 0, "head_dim must be even");
  FA4CP_CHECK_ARG(dtype == FA4CP_DTYPE_BF16 || dtype == FA4CP_DTYPE_F16,
                  "dtype must be f16 or bf16");
  if (total_q == 0) return FA4CP_OK;
  FA4CP_CHECK_ARG(out && dout && delta, "null tensor pointer");
  FA4CP_CHECK_ARG((reinterpret_cast<uintptr_t>(out) & 3u) == 0 &&
                      (reinterpret_cast<uintptr_t>(dout) & 3u) == 0,
                  "out/dout must be 4-byte aligned");
  const int64_t n_rh = total_q * num_heads_q;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned grid = elementwise_grid(n_rh * 32);
  if (dtype == FA4CP_DTYPE_BF16)
    bwd_delta_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(
        static_cast<const uint16_t*>(out), static_cast<const uint16_t*>(dout), delta, n_rh,
        head_dim);
  else
    bwd_delta_kernel<__half><<<grid, 256, 0, st>>>(static_cast<const uint16_t*>(out),
                                                   static_cast<const uint16_t*>(dout), delta,
                                                   n_rh, head_dim);
  return check_launch("attn_bwd_preprocess");
}

extern "C" int fa4cp_attn_bwd(const void* q, const void* k, const void* v, const void* dout,
                              const float* lse, const float* delta, float* dq_acc, float* dk_acc,
                              float* dv_acc, const int32_t* cu_q, const int32_t* cu_k,
                              int32_t nseq, int32_t max_seqlen_k, int64_t total_q,
                              int64_t total_k, int32_t num_heads_q, int32_t num_heads_kv,
                              int32_t head_dim, int32_t dtype, int32_t pattern, int32_t causal,
                              float softmax_scale, void* stream) {
  FA4CP_CHECK_ARG(nseq >= 1 && nseq <= 65535 && cu_q != nullptr,
                  "cu_seqlens_q must describe 1..65535 sequences");
  FA4CP_CHECK_ARG(pattern >= FA4CP_PATTERN_VARLEN && pattern <= FA4CP_PATTERN_BACK_Q,
                  "unknown pattern %d", pattern);
  FA4CP_CHECK_ARG(pattern != FA4CP_PATTERN_VARLEN || cu_k != nullptr, "cu_seqlens_k is required");
  FA4CP_CHECK_ARG(num_heads_q > 0 && num_heads_kv > 0 && num_heads_q % num_heads_kv == 0,
                  "H_q=%d not a multiple of H_kv=%d", num_heads_q, num_heads_kv);
  FA4CP_CHECK_ARG(num_heads_kv <= 65535, "too many kv heads");
  FA4CP_CHECK_ARG(total_q >= 0 && total_k >= 0 && max_seqlen_k >= 0, "bad sizes");
  FA4CP_CHECK_ARG(softmax_scale > 0.f, "softmax_scale must be positive");
  FA4CP_CHECK_ARG(dtype == FA4CP_DTYPE_BF16 || dtype == FA4CP_DTYPE_F16,
                  "the backward takes f16 or bf16 inputs");
  if (head_dim != 64 && head_dim != 128) {
    set_last_error("head_dim %d is not supported by the backward (64, 128)", head_dim);
    return FA4CP_ERR_UNSUPPORTED;
  }
  if (total_q == 0 || total_k == 0 || max_seqlen_k == 0) return FA4CP_OK;
  FA4CP_CHECK_ARG(q && k && v && dout && lse && delta && dq_acc && dk_acc && dv_acc,
                  "null tensor pointer");
  FA4CP_CHECK_ARG(al16(q) && al16(k) && al16(v) && al16(dout) && al16(dq_acc) && al16(dk_acc) &&
                      al16(dv_acc),
                  "q/k/v/dout and the accumulators must be 16-byte aligned");
  BwdParams p{};
  p.q = q;
  p.k = k;
  p.v = v;
  p.dout = dout;
  p.lse = lse;
  p.delta = delta;
  p.dq = dq_acc;
  p.dk = dk_acc;
  p.dv = dv_acc;
  p.cu_q = cu_q;
  p.cu_k = cu_k;
  p.Hq = num_heads_q;
  p.Hkv = num_heads_kv;
  p.group = num_heads_q / num_heads_kv;
  p.pattern = pattern;
  p.causal = causal ? 1 : 0;
  p.scale = softmax_scale;
  p.scale_log2 = softmax_scale * kLog2e;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == FA4CP_DTYPE_BF16)
    return head_dim == 128 ? launch_bwd<__nv_bfloat16, 128>(p, nseq, max_seqlen_k, st)
                           : launch_bwd<__nv_bfloat16, 64>(p, nseq, max_seqlen_k, st);
  return head_dim == 128 ? launch_bwd<__half, 128>(p, nseq, max_seqlen_k, st)
                         : launch_bwd<__half, 64>(p, nseq, max_seqlen_k, st);
}

extern "C" int fa4cp_convert_f32(const float* src, void* dst, int64_t n, int32_t dst_dtype,
                                 void* stream) {
  FA4CP_CHECK_ARG(n >= 0, "bad size");
  FA4CP_CHECK_ARG(dst_dtype == FA4CP_DTYPE_BF16 || dst_dtype == FA4CP_DTYPE_F16 ||
                      dst_dtype == FA4CP_DTYPE_F32,
                  "dst dtype must be f16, bf16 or f32");
  if (n == 0) return FA4CP_OK;
  FA4CP_CHECK_ARG(src && dst, "null pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned grid = elementwise_grid(n);
  if (dst_dtype == FA4CP_DTYPE_BF16)
    convert_f32_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(src, static_cast<__nv_bfloat16*>(dst), n);
  else if (dst_dtype == FA4CP_DTYPE_F16)
    convert_f32_kernel<__half><<<grid, 256, 0, st>>>(src, static_cast<__half*>(dst), n);
  else
    convert_f32_kernel<float><<<grid, 256, 0, st>>>(src, static_cast<float*>(dst), n);
  return check_launch("convert_f32");
}

extern "C" int fa4cp_add_f32(float* dst, const float* src, int64_t n, void* stream) {
  FA4CP_CHECK_ARG(n >= 0 && n % 4 == 0, "size must be a multiple of 4");
  if (n == 0) return FA4CP_OK;
  FA4CP_CHECK_ARG(dst && src && al16(dst) && al16(src), "pointers must be 16-byte aligned");
  add_f32_kernel<<<elementwise_grid(n / 4), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<float4*>(dst), reinterpret_cast<const float4*>(src), n / 4);
  return check_launch("add_f32");
}
