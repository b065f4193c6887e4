// Attention forward for sm_100a: tcgen05 MMA with TMEM accumulators, TMA-staged
// Q/K/V tiles, online softmax with one thread per query row, out + natural-log LSE.
//
// Replaces the FlashAttention-4 call of the reference (fa4_ring/fa4_backend.py:58-123)
// and, with `accumulate`, also fuses the incremental LSE merge of fa4_ring/merge.py:45-64
// into the epilogue.  The three zig-zag ring step patterns
// (fa4_ring/ring_attention.py:109-166) address their row halves in place.
//
// CTA = one (query tile of 128 rows, query head, sequence).  192 threads:
//   warps 0-3  softmax + epilogue; thread t owns query row t = TMEM lane t
//   warp  4    TMA producer (one thread): Q once, then K_j / V_j into a ring of stages
//   warp  5    TMEM allocator + MMA issuer (one thread)
// TMEM (512 columns): S0 | S1 (BN fp32 columns each, double-buffered) | O (D columns).
// P = softmax numerators overwrites the first BN*elem/4 columns of its S buffer and
// is consumed directly from TMEM as the A operand of O += P V.
// MMA issue order: S0, S1, PV0, S2, PV1, ... so the tensor core computes S_{j+1}
// while the softmax warps turn S_j into P_j.  O is rescaled lazily: only when a
// row's running max grows by more than 2^8 (log2 domain), so P <= 256.
#include <atomic>
#include <type_traits>

#include "common.cuh"

namespace fa4cp {

__device__ int g_attn_status = 0;

// SMs the persistent kernel leaves free on this host thread (set by the ring executor around
// its launches, so the K/V hop's NCCL kernel finds SMs while the attention grid runs)
thread_local int t_sm_reserve = 0;
void set_sm_reserve(int n) { t_sm_reserve = n > 0 ? n : 0; }

// bound of the ring kernel's wait for a hop counter written by a peer (fa4cp_ring_set_wait_timeout_ms)
std::atomic<int> g_ring_wait_ms{10000};

namespace {

constexpr int BM = 128;
constexpr int kThreads = 192;
constexpr float kNegInf = -__builtin_huge_valf();
constexpr float kRescaleThreshold = 8.0f;  // log2 units

// codes written to the device status word when a bounded wait gives up
enum : int {
  kErrQ = 0x101, kErrKEmpty, kErrVEmpty, kErrKFull, kErrPFull, kErrVFull,
  kErrSFull, kErrODone, kErrDrain
};

struct Params {
  const int32_t* cu_q;
  const int32_t* cu_k;
  void* out;
  float* lse;
  const float* q_descale;
  const float* k_descale;
  const float* v_descale;
  int nseq, n_qtiles, Hq, Hkv, group;
  int pattern, causal, accumulate;
  int in_fmt;    // kind::f16 operand format: 0 f16, 1 bf16 (unused for e4m3)
  int out_bf16;  // 1 -> bf16 output, 0 -> f16 output
  float scale_log2;
  int n_tiles;  // persistent kernel: tiles of the whole schedule (tile_work decodes them)
  // self-test only (fa4cp_selftest_wait_expiry): index of the KV tile whose K copy the
  // producer never issues, so the consumer's bounded wait must expire; -1 otherwise
  int debug_withhold_kv;
  // paged K/V (two-tile kernel, VARLEN pattern): K/V rows of sequence j at logical row r live
  // in page block_table[j * max_pages + r / page_size], row r % page_size of the page pool
  // [pages, page_size, Hkv, D]; nullptr: contiguous K/V at cu_k
  const int32_t* block_table;
  int page_size, max_pages;
};

template <int D_, int BN_, int STAGES_, bool FP8_>
struct Traits {
  static constexpr int D = D_, BN = BN_, STAGES = STAGES_;
  static constexpr bool FP8 = FP8_;
  static constexpr int ELEM = FP8 ? 1 : 2;
  static constexpr int CHUNK = 128 / ELEM;  // elements of one 128-byte swizzle row
  static constexpr int NCH = D / CHUNK;     // 128-byte column blocks along D
  static constexpr int MMA_K = FP8 ? 32 : 16;
  static constexpr int Q_BYTES = BM * D * ELEM;
  static constexpr int KV_BYTES = BN * D * ELEM;
  static constexpr int Q_CHUNK_BYTES = BM * 128;
  static constexpr int KV_CHUNK_BYTES = BN * 128;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + Q_BYTES;
  static constexpr int OFF_V = OFF_K + STAGES * KV_BYTES;
  static constexpr int OFF_BAR = OFF_V + STAGES * KV_BYTES;
  // q_full, k_full[S], k_empty[S], v_full[S], v_empty[S], s_full[2], p_full[2], o_done[2], teardown
  static constexpr int NUM_BARS = 1 + 4 * STAGES + 2 + 2 + 2 + 1;
  static constexpr int SMEM_BYTES = OFF_BAR + NUM_BARS * 8 + 16 + 1024;
  static constexpr int TM_O = 2 * BN;
  static constexpr int TM_COLS = 512;
  // P columns per S buffer: 32-bit columns holding BN values of ELEM bytes
  static constexpr int P_COLS = BN * ELEM / 4;
  static_assert(D % CHUNK == 0, "head_dim must be a multiple of one 128-byte swizzle row");
  static_assert(2 * BN + D <= TM_COLS, "TMEM budget");
  static_assert(BN % 32 == 0 && D % 32 == 0, "tile shape");
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
};

struct Geometry {
  int q_start, q_len, k_start, k_len;
};

// CTA order (blockIdx.x, one sequence per blockIdx.z): q-tiles are taken in chunks of
// kQtileChunk, heaviest (latest, under causal masking) chunk first; inside a chunk all
// CTAs of one kv head run before the next kv head's, q-tile major, q head minor.  The
// CTAs resident at any time then read the K/V of only a few kv heads, which stay in L2
// instead of every kv head's K/V streaming through it.  Each chunk reads the K/V of every
// kv head once more (a kv head's CTAs of the next chunk start after all other kv heads' K/V
// went through L2), so the chunk sets the K/V re-reads: measured on the two-tile kernel,
// causal bf16 N=32768 Hq=32 Hkv=8 D=128, DRAM traffic 1.67x the algorithmic bytes with
// chunks of 16 pairs, 1.22x with 32, 1.05x with 64, 0.97x with one chunk, at equal kernel
// time; a single chunk slowed the persistent e4m3 kernel by 3% (its heavy-first balance).
constexpr int kQtileChunk = 64;

__device__ __forceinline__ bool cta_tile(const Params& p, int& head, int& qtile) {
  const int ch = min(kQtileChunk, p.n_qtiles);
  const int per_chunk = p.Hkv * ch * p.group;
  const int L = int(blockIdx.x);
  const int chunk = L / per_chunk;
  const int r = L - chunk * per_chunk;
  const int kvh = r / (ch * p.group);
  const int r2 = r - kvh * (ch * p.group);
  const int qt_desc = chunk * ch + r2 / p.group;
  if (qt_desc >= p.n_qtiles) return false;  // padding of the last chunk
  head = kvh * p.group + (r2 % p.group);
  qtile = p.n_qtiles - 1 - qt_desc;
  return true;
}

inline unsigned cta_grid_x(int n_qtiles, int Hq) {
  const int ch = n_qtiles < kQtileChunk ? n_qtiles : kQtileChunk;
  const int chunks = (n_qtiles + ch - 1) / ch;
  return unsigned(chunks * ch * Hq);
}

__device__ __forceinline__ Geometry seq_geometry(const Params& p, int seq) {
  Geometry g;
  const int a = p.cu_q[seq], b = p.cu_q[seq + 1];
  if (p.pattern == FA4CP_PATTERN_VARLEN) {
    g.q_start = a;
    g.q_len = b - a;
    g.k_start = p.cu_k[seq];
    g.k_len = p.cu_k[seq + 1] - g.k_start;
  } else {
    const int n = b - a, hh = n / 2;
    if (p.pattern == FA4CP_PATTERN_FRONT_KV) {
      g.q_start = a; g.q_len = n; g.k_start = a; g.k_len = hh;
    } else {  // FA4CP_PATTERN_BACK_Q
      g.q_start = a + hh; g.q_len = n - hh; g.k_start = a; g.k_len = n;
    }
  }
  return g;
}

template <class TR>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const Params p) {
  constexpr int D = TR::D, BN = TR::BN, ST = TR::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int head, qtile;
  if (!cta_tile(p, head, qtile)) return;  // uniform for the whole CTA
  const int seq = blockIdx.z;

  const Geometry g = seq_geometry(p, seq);
  const int q0 = qtile * BM;
  if (q0 >= g.q_len) return;  // uniform for the whole CTA, before any setup
  const int rows = min(BM, g.q_len - q0);
  const int diag = g.k_len - g.q_len;  // causal: key j visible to row i iff j <= i + diag
  int kv_end = g.k_len;
  if (p.causal) kv_end = min(g.k_len, q0 + rows + diag);
  const int n_kv = kv_end > 0 ? (kv_end + BN - 1) / BN : 0;
  const int kvh = head / p.group;

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + TR::OFF_BAR);
  const uint32_t bar0 = smem_u32(bars);
  auto BAR = [&](int i) -> uint32_t { return bar0 + 8u * uint32_t(i); };
  const uint32_t q_full = BAR(0);
  auto k_full = [&](int s) { return BAR(1 + s); };
  auto k_empty = [&](int s) { return BAR(1 + ST + s); };
  auto v_full = [&](int s) { return BAR(1 + 2 * ST + s); };
  auto v_empty = [&](int s) { return BAR(1 + 3 * ST + s); };
  auto s_full = [&](int b) { return BAR(1 + 4 * ST + b); };
  auto p_full = [&](int b) { return BAR(3 + 4 * ST + b); };
  // PV_i commits o_done(i & 1): a waiter for PV_i is then never two phases away
  // from the barrier's current phase (PV_{i-2} is known complete, PV_{i+2} cannot
  // have been issued), so parity waits are exact.
  auto o_done = [&](int b) { return BAR(5 + 4 * ST + b); };
  const uint32_t td_bar = BAR(7 + 4 * ST);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + TR::NUM_BARS);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* status = &g_attn_status;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < ST; ++s) {
      mbar_init(k_full(s), 1);
      mbar_init(k_empty(s), 1);
      mbar_init(v_full(s), 1);
      mbar_init(v_empty(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(s_full(b), 1);
      mbar_init(p_full(b), 128);
    }
    mbar_init(o_done(0), 1);
    mbar_init(o_done(1), 1);
    mbar_init(td_bar, 1);
    *abort = 0;
    fence_mbar_init();
  }
  if (warp == 4 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 5) {
    tmem_alloc(smem_u32(tmem_slot), TR::TM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 4) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const uint64_t pol_kv = policy_evict_last();
      int last_k[ST], last_v[ST];
      for (int s = 0; s < ST; ++s) last_k[s] = last_v[s] = -1;
      mbar_arrive_expect_tx(q_full, TR::Q_BYTES);
#pragma unroll
      for (int c = 0; c < TR::NCH; ++c)
        tma_load_3d(smem_u32(smem + TR::OFF_Q + c * TR::Q_CHUNK_BYTES), &tmQ, c * TR::CHUNK, head,
                    g.q_start + q0, q_full);
      for (int j = 0; j < n_kv; ++j) {
        const int s = j % ST, ph = (j / ST) & 1;
        const int row = g.k_start + j * BN;
        if (j >= ST && !mbar_wait(k_empty(s), ph ^ 1, abort, kErrKEmpty, status)) break;
        if (j != p.debug_withhold_kv) {
          mbar_arrive_expect_tx(k_full(s), TR::KV_BYTES);
#pragma unroll
          for (int c = 0; c < TR::NCH; ++c)
            tma_load_3d_hint(smem_u32(smem + TR::OFF_K + s * TR::KV_BYTES + c * TR::KV_CHUNK_BYTES),
                             &tmK, c * TR::CHUNK, kvh, row, k_full(s), pol_kv);
          last_k[s] = j;
        }
        if (j >= ST && !mbar_wait(v_empty(s), ph ^ 1, abort, kErrVEmpty, status)) break;
        mbar_arrive_expect_tx(v_full(s), TR::KV_BYTES);
#pragma unroll
        for (int c = 0; c < TR::NCH; ++c)
          tma_load_3d_hint(smem_u32(smem + TR::OFF_V + s * TR::KV_BYTES + c * TR::KV_CHUNK_BYTES),
                           &tmV, c * TR::CHUNK, kvh, row, v_full(s), pol_kv);
        last_v[s] = j;
      }
      {
        // every copy this thread issued has landed before it leaves its role (on the
        // normal path the consumers already waited for them, so this returns at once)
        mbar_wait_drain(q_full, 0, kErrDrain, status);
        for (int s = 0; s < ST; ++s) {
          if (last_k[s] >= 0) mbar_wait_drain(k_full(s), (last_k[s] / ST) & 1, kErrDrain, status);
          if (last_v[s] >= 0) mbar_wait_drain(v_full(s), (last_v[s] / ST) & 1, kErrDrain, status);
        }
      }
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const int fmt = TR::FP8 ? 0 : p.in_fmt;
      const uint32_t idesc_qk = make_idesc(BM, BN, fmt, fmt, 0, 0);
      const uint32_t idesc_pv = make_idesc(BM, D, fmt, fmt, 0, 1);
      const uint32_t sQ = smem_u32(smem + TR::OFF_Q);
      auto issue_pv = [&](int i) -> bool {
        const int s = i % ST, b = i & 1;
        if (!mbar_wait(p_full(b), (i >> 1) & 1, abort, kErrPFull, status)) return false;
        if (!mbar_wait(v_full(s), (i / ST) & 1, abort, kErrVFull, status)) return false;
        tc_fence_after();
        const uint32_t sV = smem_u32(smem + TR::OFF_V + s * TR::KV_BYTES);
#pragma unroll
        for (int kk = 0; kk < BN / TR::MMA_K; ++kk) {
          const uint64_t bdesc = make_desc_sw128(sV + kk * TR::MMA_K * 128, TR::KV_CHUNK_BYTES, 1024);
          const uint32_t a_tmem = tmem + uint32_t(b * BN + kk * 8);
          if constexpr (TR::FP8)
            mma_f8_ts(tmem + TR::TM_O, a_tmem, bdesc, idesc_pv, (i > 0 || kk > 0) ? 1u : 0u);
          else
            mma_f16_ts(tmem + TR::TM_O, a_tmem, bdesc, idesc_pv, (i > 0 || kk > 0) ? 1u : 0u);
        }
        tc_commit(o_done(b));
        tc_commit(v_empty(s));
        return true;
      };
      bool ok = mbar_wait(q_full, 0, abort, kErrQ, status);
      tc_fence_after();
      for (int j = 0; ok && j < n_kv; ++j) {
        const int s = j % ST, b = j & 1;
        if (!mbar_wait(k_full(s), (j / ST) & 1, abort, kErrKFull, status)) { ok = false; break; }
        tc_fence_after();
        const uint32_t sK = smem_u32(smem + TR::OFF_K + s * TR::KV_BYTES);
#pragma unroll
        for (int kk = 0; kk < D / TR::MMA_K; ++kk) {
          const int off = kk * 32;  // bytes along D of this K-step
          const uint32_t ca = (off / 128) * TR::Q_CHUNK_BYTES + (off % 128);
          const uint32_t cb = (off / 128) * TR::KV_CHUNK_BYTES + (off % 128);
          const uint64_t adesc = make_desc_sw128(sQ + ca, 16, 1024);
          const uint64_t bdesc = make_desc_sw128(sK + cb, 16, 1024);
          if constexpr (TR::FP8)
            mma_f8_ss(tmem + uint32_t(b * BN), adesc, bdesc, idesc_qk, kk > 0 ? 1u : 0u);
          else
            mma_f16_ss(tmem + uint32_t(b * BN), adesc, bdesc, idesc_qk, kk > 0 ? 1u : 0u);
        }
        tc_commit(s_full(b));
        tc_commit(k_empty(s));
        if (j > 0 && !issue_pv(j - 1)) { ok = false; break; }
      }
      if (ok && n_kv > 0) issue_pv(n_kv - 1);
      // every MMA issued above has completed before TMEM is released
      tc_commit(td_bar);
      mbar_wait_drain(td_bar, 0, kErrDrain, status);
    }
  } else {
    // ------------------------------------------------------------ softmax + epilogue
    const int r = warp * 32 + lane;
    const uint32_t t_lane = tmem + (uint32_t(warp * 32) << 16);
    const int key_lim = q0 + r + diag;
    float scale = p.scale_log2;
    float vscale = 1.0f;
    if (p.q_descale) scale *= p.q_descale[kvh];
    if (p.k_descale) scale *= p.k_descale[kvh];
    if (p.v_descale) vscale = p.v_descale[kvh];
    float m = kNegInf, l = 0.f;
    bool aborted = false;

    for (int j = 0; j < n_kv; ++j) {
      const int b = j & 1;
      bool ok = mbar_wait(s_full(b), (j >> 1) & 1, abort, kErrSFull, status);
      if (!__all_sync(0xffffffffu, ok)) { aborted = true; break; }
      tc_fence_after();
      uint32_t sr[BN / 32][32];
#pragma unroll
      for (int c = 0; c < BN / 32; ++c) tmem_ld32(t_lane + uint32_t(b * BN + c * 32), sr[c]);
      tmem_wait_ld();
#pragma unroll
      for (int c = 0; c < BN / 32; ++c) reg_fence32(sr[c]);

      const int kbase = j * BN;
      const bool need_mask = (kbase + BN > g.k_len) || (p.causal && kbase + BN - 1 > q0 + diag);
      if (need_mask) {
#pragma unroll
        for (int c = 0; c < BN / 32; ++c)
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const int key = kbase + c * 32 + e;
            if (key >= g.k_len || (p.causal && key > key_lim)) sr[c][e] = __float_as_uint(kNegInf);
          }
      }
      float mx = kNegInf;
#pragma unroll
      for (int c = 0; c < BN / 32; ++c)
#pragma unroll
        for (int e = 0; e < 32; ++e) mx = fmaxf(mx, __uint_as_float(sr[c][e]));
      const float m_new = fmaxf(m, mx);
      if (j == 0) {
        m = m_new;
      } else {
        const bool need = (m_new - m) * scale > kRescaleThreshold;
        if (__any_sync(0xffffffffu, need)) {
          const float f = need ? ex2_approx((m - m_new) * scale) : 1.0f;
          if (need) { l *= f; m = m_new; }
          ok = mbar_wait(o_done((j - 1) & 1), ((j - 1) >> 1) & 1, abort, kErrODone, status);
          if (!__all_sync(0xffffffffu, ok)) { aborted = true; break; }
          tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < D / 32; ++c) {
            uint32_t o[32];
            tmem_ld32(t_lane + uint32_t(TR::TM_O + c * 32), o);
            tmem_wait_ld();
            reg_fence32(o);
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * f);
            tmem_st32(t_lane + uint32_t(TR::TM_O + c * 32), o);
          }
          tmem_wait_st();
        }
      }
      const float neg_m = (m == kNegInf) ? 0.f : -m * scale;
      float rs = 0.f;
      if constexpr (TR::FP8) {
        uint32_t pw[32];
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) {
#pragma unroll
          for (int e = 0; e < 32; e += 4) {
            float x0 = ex2_approx(fmaf(__uint_as_float(sr[c][e + 0]), scale, neg_m));
            float x1 = ex2_approx(fmaf(__uint_as_float(sr[c][e + 1]), scale, neg_m));
            float x2 = ex2_approx(fmaf(__uint_as_float(sr[c][e + 2]), scale, neg_m));
            float x3 = ex2_approx(fmaf(__uint_as_float(sr[c][e + 3]), scale, neg_m));
            rs += (x0 + x1) + (x2 + x3);
            pw[(c * 32 + e) / 4] = pack_e4m3x4(x0, x1, x2, x3);
          }
        }
        static_assert(!TR::FP8 || BN == 128, "FP8 P store assumes 128 keys (32 columns)");
        tmem_st32(t_lane + uint32_t(b * BN), pw);
      } else {
#pragma unroll
        for (int half = 0; half < BN / 64; ++half) {
          uint32_t pw[32];
#pragma unroll
          for (int e = 0; e < 64; e += 2) {
            const int c = half * 2 + (e >> 5), ee = e & 31;
            float x0 = ex2_approx(fmaf(__uint_as_float(sr[c][ee]), scale, neg_m));
            float x1 = ex2_approx(fmaf(__uint_as_float(sr[c][ee + 1]), scale, neg_m));
            rs += x0 + x1;
            pw[e >> 1] = p.in_fmt ? pack_bf16x2(x0, x1) : pack_f16x2(x0, x1);
          }
          tmem_st32(t_lane + uint32_t(b * BN + half * 32), pw);
        }
      }
      l += rs;
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(p_full(b));
    }

    // ------------------------------------------------------------ epilogue
    if (!aborted && n_kv > 0) {
      bool ok = mbar_wait(o_done((n_kv - 1) & 1), ((n_kv - 1) >> 1) & 1, abort, kErrODone, status);
      if (!__all_sync(0xffffffffu, ok)) aborted = true;
      tc_fence_after();
    }
    if (!aborted) {
      const bool valid = r < rows;
      const int64_t grow = int64_t(g.q_start) + q0 + r;
      const float lse_new = (l > 0.f) ? (m * scale + lg2_approx(l)) * kLn2 : kNegInf;
      float* lse_ptr = p.lse + grow * p.Hq + head;
      // output coefficients: out = acc * ca + O_raw * cb
      float ca = 0.f, cb = (l > 0.f) ? vscale / l : 0.f, lse_out = lse_new;
      bool write = valid;
      bool read_acc = false;
      if (valid && p.accumulate) {
        const float acc_lse = *lse_ptr;
        if (lse_new == kNegInf) {
          write = false;  // this partial covers nothing for the row
        } else if (acc_lse != kNegInf) {
          const float mm = fmaxf(acc_lse, lse_new);
          const float wa = ex2_approx((acc_lse - mm) * kLog2e);
          const float wb = ex2_approx((lse_new - mm) * kLog2e);
          const float inv = 1.0f / (wa + wb);
          ca = wa * inv;
          cb *= wb * inv;
          lse_out = mm + lg2_approx(wa + wb) * kLn2;
          read_acc = true;
        }
      }
      uint8_t* orow = static_cast<uint8_t*>(p.out) + (grow * p.Hq + head) * int64_t(D) * 2;
      const bool has_o = n_kv > 0;  // CTA-uniform
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        if (has_o) {
          tmem_ld32(t_lane + uint32_t(TR::TM_O + c * 32), o);
          tmem_wait_ld();
          reg_fence32(o);
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = 0u;
        }
        if (write) {
          uint4* dst = reinterpret_cast<uint4*>(orow + c * 64);
          float f[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) f[e] = has_o ? __uint_as_float(o[e]) * cb : 0.f;
          if (read_acc) {
#pragma unroll
            for (int v4 = 0; v4 < 4; ++v4) {
              const uint4 a = dst[v4];
              const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                float lo, hi;
                if (p.out_bf16) {
                  lo = __uint_as_float(w[i] << 16);
                  hi = __uint_as_float(w[i] & 0xFFFF0000u);
                } else {
                  const float2 t = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
                  lo = t.x; hi = t.y;
                }
                f[v4 * 8 + 2 * i] = fmaf(lo, ca, f[v4 * 8 + 2 * i]);
                f[v4 * 8 + 2 * i + 1] = fmaf(hi, ca, f[v4 * 8 + 2 * i + 1]);
              }
            }
          }
#pragma unroll
          for (int v4 = 0; v4 < 4; ++v4) {
            uint32_t w[4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
              w[i] = p.out_bf16 ? pack_bf16x2(f[v4 * 8 + 2 * i], f[v4 * 8 + 2 * i + 1])
                                : pack_f16x2(f[v4 * 8 + 2 * i], f[v4 * 8 + 2 * i + 1]);
            dst[v4] = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
      }
      if (write) *lse_ptr = lse_out;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 5) tmem_dealloc(tmem, TR::TM_COLS);
}

// ---------------------------------------------------------------------------
// v2: two query tiles per CTA, two softmax warpgroups ping-ponging on the tensor core
// ---------------------------------------------------------------------------
// CTA = rows [q0, q0 + 256) of one (head, sequence): tile 0 = first 128 rows, tile 1 =
// next 128.  Both tiles share every K/V tile staged in shared memory.  384 threads:
//   warps 0-3  softmax + epilogue of tile 0      warps 4-7  softmax + epilogue of tile 1
//   warp  8    TMA producer                      warp  9    TMEM allocator + MMA issuer
//   warps 10-11 idle (complete the producer warpgroup for the register re-split)
// Registers: launched at 168/thread (384 x 168 = 64512); the producer warpgroup drops to
// 72 (104 when persistent) and each softmax warpgroup rises to 216 (200):
// 128 x (216 + 216 + 72) = 128 x (200 + 200 + 104) = 64512.
// TMEM: S0 | S1 (BN fp32 columns each) | O0 | O1 (D columns each).  One S buffer per
// tile: S_t(j+1) is issued after PV_t(j), so the completion of S_t(j+1) also proves
// PV_t(j) finished -- a softmax warpgroup may rescale O_t right after its s_full wait.
// MMA order per KV tile j:  PV0(j) S0(j+1) PV1(j) S1(j+1): while warpgroup 0 turns
// S0(j+1) into P0(j+1), the tensor core runs PV1(j) and S1(j+1), and vice versa.
#ifndef FA4CP_EXP2_EMU_PER_8
#define FA4CP_EXP2_EMU_PER_8 0
#endif
#ifndef FA4CP_EXP2_EMU_FP8
#define FA4CP_EXP2_EMU_FP8 0
#endif
#ifndef FA4CP_P_SPLIT
#define FA4CP_P_SPLIT 1
#endif
// register re-split (setmaxnreg) of the two-tile kernel: softmax warpgroups / the warpgroup
// of the producer and MMA warps, persistent (P) and one-tile (NP) forms
#ifndef FA4CP_REGS_SOFTMAX_P
#define FA4CP_REGS_SOFTMAX_P 200
#endif
#ifndef FA4CP_REGS_PRODUCER_P
#define FA4CP_REGS_PRODUCER_P 104
#endif
#ifndef FA4CP_REGS_SOFTMAX_NP
#define FA4CP_REGS_SOFTMAX_NP 216
#endif
#ifndef FA4CP_REGS_PRODUCER_NP
#define FA4CP_REGS_PRODUCER_NP 72
#endif

template <int D_, int BN_, int STAGES_, bool FP8_, int PERSIST_ = -1>
struct Traits2 {
  static constexpr int D = D_, BN = BN_, STAGES = STAGES_;
  static constexpr bool FP8 = FP8_;
  // of every 8 element pairs of P, this many take exp2 on the FMA pipe (exp2_poly_x2)
  // and the rest on the MUFU unit, balancing the two pipes against the tensor core
  static constexpr int EXP2_EMU_PER_8 = FP8 ? FA4CP_EXP2_EMU_FP8 : FA4CP_EXP2_EMU_PER_8;
  // P is handed to the MMA warp in this many key slices (one barrier each), so the PV
  // MMAs of the first slice run while the softmax warpgroup finishes the rest
  static constexpr int P_SPLIT = FA4CP_P_SPLIT;
  static constexpr int ELEM = FP8 ? 1 : 2;
  static constexpr int CHUNK = 128 / ELEM;
  static constexpr int NCH = D / CHUNK;
  static constexpr int MMA_K = FP8 ? 32 : 16;
  static constexpr int Q_TILE_BYTES = BM * D * ELEM;
  static constexpr int KV_BYTES = BN * D * ELEM;
  static constexpr int Q_CHUNK_BYTES = BM * 128;
  static constexpr int KV_CHUNK_BYTES = BN * 128;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = 2 * Q_TILE_BYTES;
  static constexpr int OFF_V = OFF_K + STAGES * KV_BYTES;
  static constexpr int OFF_BAR = OFF_V + STAGES * KV_BYTES;
  // q_full, k_full[S], k_empty[S], v_full[S], v_empty[S], s_full[2], o_done[2], teardown,
  // q_empty, o_free[2], p_full[2][P_SPLIT]
  static constexpr int NUM_BARS = 1 + 4 * STAGES + 2 + 2 + 1 + 1 + 2 + 2 * FA4CP_P_SPLIT;
  static constexpr int SMEM_BYTES = OFF_BAR + NUM_BARS * 8 + 16 + 1024;
  static constexpr int TM_COLS = 512;
  static constexpr int THREADS = 384;
  // FP8 runs persistently (one CTA per SM walking the tile schedule: its MMAs take half the
  // time, so per-CTA set-up and epilogue weigh twice as much); f16/bf16 measured faster with
  // one CTA per tile, where the tile loop has a single trip and its cross-tile state folds
  // away, leaving the softmax warpgroups 216 registers.
  static constexpr bool PERSISTENT = PERSIST_ < 0 ? FP8 : PERSIST_ != 0;
  static constexpr int REGS_SOFTMAX = PERSISTENT ? FA4CP_REGS_SOFTMAX_P : FA4CP_REGS_SOFTMAX_NP;
  static constexpr int REGS_PRODUCER = PERSISTENT ? FA4CP_REGS_PRODUCER_P : FA4CP_REGS_PRODUCER_NP;
  static_assert(128 * (2 * REGS_SOFTMAX + REGS_PRODUCER) <= THREADS * 168,
                "register re-split exceeds the launch allocation");
  __host__ __device__ static constexpr int tm_s(int t) { return t * BN; }
  __host__ __device__ static constexpr int tm_o(int t) { return 2 * BN + t * D; }
  static_assert(D % CHUNK == 0, "head_dim must be a multiple of one 128-byte swizzle row");
  static_assert(2 * BN + 2 * D <= TM_COLS, "TMEM budget");
  static_assert(BN == 128, "softmax register layout assumes 128 keys per tile");
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
};

// One unit of work of the persistent kernel: 2 x 128 query rows of one (head, sequence).
struct TileWork {
  Geometry g;
  int seq, head, kvh, q0, diag, nmax;
  int rows_t[2], n_t[2];
};

// Tile `tile` of the persistent schedule.  Order: chunks of kQtileChunk query-tile pairs,
// heaviest (latest) chunk first across all sequences; inside a chunk, sequence, then kv
// head, then query-tile pair, then query head of the GQA group -- so the tiles in flight
// at any time touch the K/V of few kv heads (which then stay in L2) and heavy causal tiles
// are scheduled before light ones.  Returns false for padding / past-the-end tiles.
__device__ __forceinline__ bool tile_work(const Params& p, int tile, int BN, TileWork& w) {
  const int ch = min(kQtileChunk, p.n_qtiles);
  const int per_seq = ch * p.Hq;
  const int per_chunk = per_seq * p.nseq;
  const int chunk = tile / per_chunk;
  int r = tile - chunk * per_chunk;
  const int seq = r / per_seq;
  r -= seq * per_seq;
  const int kvh = r / (ch * p.group);
  const int r2 = r - kvh * (ch * p.group);
  const int qt_desc = chunk * ch + r2 / p.group;
  if (qt_desc >= p.n_qtiles) return false;
  w.head = kvh * p.group + r2 % p.group;
  w.kvh = kvh;
  w.seq = seq;
  w.g = seq_geometry(p, seq);
  w.q0 = (p.n_qtiles - 1 - qt_desc) * 2 * BM;
  if (w.q0 >= w.g.q_len) return false;
  w.diag = w.g.k_len - w.g.q_len;
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const int first = w.q0 + t * BM;
    w.rows_t[t] = max(0, min(BM, w.g.q_len - first));
    int kv_end = w.g.k_len;
    if (p.causal) kv_end = min(w.g.k_len, first + w.rows_t[t] + w.diag);
    w.n_t[t] = (w.rows_t[t] > 0 && kv_end > 0) ? (kv_end + BN - 1) / BN : 0;
  }
  w.nmax = max(w.n_t[0], w.n_t[1]);
  return true;
}

// e4m3 only: the first K/V tile of query tile t goes to the PV MMA as two e4m3 terms
// (fp8_p_to_tmem) when some row of the tile sees fewer than 128 keys in all -- causal: its
// first row; otherwise every row sees k_len keys.  Such a row's keys all lie in that tile,
// and over few keys the rounding of an e4m3 P does not average out; a row with 128 or more
// keys needs no split.  Only tiles at the start of a short key range qualify, so the extra
// MMAs (measured 3% when every causal diagonal tile was split, cfg3 N=131072) vanish.  The
// softmax warps and the MMA warp evaluate it alike.
__device__ __forceinline__ bool fp8_split_first(const Params& p, const TileWork& w, int t) {
  return p.causal ? (w.q0 + t * BM + w.diag + 1 < 128) : (w.g.k_len < 128);
}

inline int persistent_tiles(int n_qtiles, int Hq, int nseq) {
  const int ch = n_qtiles < kQtileChunk ? n_qtiles : kQtileChunk;
  return (n_qtiles + ch - 1) / ch * ch * Hq * nseq;
}

// exp2 of one element pair: the pair index decides, at compile time, which pipe does it
template <class TR>
__device__ __forceinline__ uint64_t exp2_pair(int pair, uint64_t x) {
  if ((pair & 7) < TR::EXP2_EMU_PER_8) return TR::FP8 ? exp2_poly2_x2(x) : exp2_poly_x2(x);
  return f2pack(ex2_approx(f2lo(x)), ex2_approx(f2hi(x)));
}

// e4m3 P of one 128-key tile into TMEM, the A operand of the PV MMA.  x = exp2(S * scale - m)
// per key; hi = e4m3(x) goes to the 32 columns at `taddr`.  With SPLIT, lo = e4m3(x - hi)
// goes to the next 32 columns and the MMA warp runs that tile's PV MMA twice (hi, then lo),
// so P carries about 7 significant bits instead of 4 (|hi + lo - x| <= 0.002 max(x, 1) against
// 0.06 max(x, 1) for hi alone).  The kernels split the tiles of rows that see fewer than 128
// keys in all: over few keys the rounding of P does not average out (a row seeing 2 keys errs
// by up to ~0.03 |v| with hi alone).  Returns the fp32 row sum of x (a pair).
// SPLIT is a template argument: the callers compile their per-tile softmax step twice and
// run the split tiles outside the loop over the common ones (a branch inside the step
// measured slower on the unsplit tiles).
template <class TR, bool SPLIT>
__device__ __forceinline__ uint64_t fp8_p_to_tmem(uint32_t (&sr)[TR::BN / 32][32], uint64_t scale2,
                                                  uint64_t negm2, uint32_t taddr) {
  static_assert(TR::FP8 && TR::BN == 128, "e4m3 P of 128 keys (32 TMEM columns)");
  uint64_t rs2[2] = {0ull, 0ull};
  if constexpr (!SPLIT) {
    uint32_t pw[32];
#pragma unroll
    for (int c = 0; c < TR::BN / 32; ++c) {
#pragma unroll
      for (int e = 0; e < 32; e += 4) {
        const uint64_t a = ffma2(f2pack(__uint_as_float(sr[c][e]), __uint_as_float(sr[c][e + 1])), scale2, negm2);
        const uint64_t b = ffma2(f2pack(__uint_as_float(sr[c][e + 2]), __uint_as_float(sr[c][e + 3])), scale2, negm2);
        const uint64_t ea = exp2_pair<TR>((c * 32 + e) / 2, a);
        const uint64_t eb = exp2_pair<TR>((c * 32 + e) / 2 + 1, b);
        rs2[0] = fadd2(rs2[0], ea);
        rs2[1] = fadd2(rs2[1], eb);
        pw[(c * 32 + e) / 4] = pack_e4m3x4(f2lo(ea), f2hi(ea), f2lo(eb), f2hi(eb));
      }
    }
    tmem_st32(taddr, pw);
  } else {
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {  // 64 keys at a time: 16 columns of hi, 16 of lo
      uint32_t hi[16], lo[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int key = hf * 64 + 4 * i, c = key >> 5, e = key & 31;
        const uint64_t a = ffma2(f2pack(__uint_as_float(sr[c][e]), __uint_as_float(sr[c][e + 1])), scale2, negm2);
        const uint64_t b = ffma2(f2pack(__uint_as_float(sr[c][e + 2]), __uint_as_float(sr[c][e + 3])), scale2, negm2);
        const uint64_t ea = exp2_pair<TR>(key / 2, a);
        const uint64_t eb = exp2_pair<TR>(key / 2 + 1, b);
        rs2[0] = fadd2(rs2[0], ea);
        rs2[1] = fadd2(rs2[1], eb);
        hi[i] = pack_e4m3x4(f2lo(ea), f2hi(ea), f2lo(eb), f2hi(eb));
        float h0, h1, h2, h3;
        unpack_e4m3x4(hi[i], h0, h1, h2, h3);
        lo[i] = pack_e4m3x4(f2lo(ea) - h0, f2hi(ea) - h1, f2lo(eb) - h2, f2hi(eb) - h3);
      }
      tmem_st16(taddr + uint32_t(hf * 16), hi);
      tmem_st16(taddr + uint32_t(32 + hf * 16), lo);
    }
  }
  return fadd2(rs2[0], rs2[1]);
}

template <class TR>
__global__ void __launch_bounds__(TR::THREADS, 1)
    attn_fwd_2q_kernel(const __grid_constant__ CUtensorMap tmQ,
                       const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const Params p) {
  constexpr int D = TR::D, BN = TR::BN, ST = TR::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + TR::OFF_BAR);
  const uint32_t bar0 = smem_u32(bars);
  auto BAR = [&](int i) -> uint32_t { return bar0 + 8u * uint32_t(i); };
  const uint32_t q_full = BAR(0);
  auto k_full = [&](int s) { return BAR(1 + s); };
  auto k_empty = [&](int s) { return BAR(1 + ST + s); };
  auto v_full = [&](int s) { return BAR(1 + 2 * ST + s); };
  auto v_empty = [&](int s) { return BAR(1 + 3 * ST + s); };
  auto s_full = [&](int t) { return BAR(1 + 4 * ST + t); };
  auto o_done = [&](int t) { return BAR(3 + 4 * ST + t); };
  const uint32_t td_bar = BAR(5 + 4 * ST);
  const uint32_t q_empty = BAR(6 + 4 * ST);
  auto o_free = [&](int t) { return BAR(7 + 4 * ST + t); };
  auto p_full = [&](int t, int h) { return BAR(9 + 4 * ST + t * TR::P_SPLIT + h); };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + TR::NUM_BARS);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* status = &g_attn_status;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int s = 0; s < ST; ++s) {
      mbar_init(k_full(s), 1);
      mbar_init(k_empty(s), 1);
      mbar_init(v_full(s), 1);
      mbar_init(v_empty(s), 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(s_full(t), 1);
      for (int h = 0; h < TR::P_SPLIT; ++h) mbar_init(p_full(t, h), 128);
      mbar_init(o_done(t), 1);
      mbar_init(o_free(t), 128);
    }
    mbar_init(td_bar, 1);
    *abort = 0;
    fence_mbar_init();
  }
  if (warp == 8 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 9) {
    tmem_alloc(smem_u32(tmem_slot), TR::TM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int n_tiles = p.n_tiles;
  // static boustrophedon schedule: round k takes tiles [k*G, (k+1)*G), forward on even
  // rounds and backward on odd ones, so with heaviest-first tiles every CTA pairs heavy
  // and light tiles (the same sequence for all roles of the CTA)
  const int G = int(gridDim.x);
  auto snake_tile = [&](int k) -> int {
    return k * G + ((k & 1) ? G - 1 - int(blockIdx.x) : int(blockIdx.x));
  };

  if (warp >= 8) {
   setmaxnreg_dec<TR::REGS_PRODUCER>();
   if (warp == 8) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const uint64_t pol_kv = policy_evict_last();
      int last_k[ST], last_v[ST];
      for (int s = 0; s < ST; ++s) last_k[s] = last_v[s] = -1;
      int kv_it = 0, tile_it = 0;
      bool ok = true;
      for (int it_tile = 0, tile = snake_tile(0); (TR::PERSISTENT || it_tile == 0) && ok && tile < n_tiles; tile = snake_tile(++it_tile)) {
        TileWork w;
        if (!tile_work(p, tile, BN, w)) continue;
        // the Q buffers are free once every S MMA of the previous tile has completed
        if (tile_it > 0 && !mbar_wait(q_empty, (tile_it - 1) & 1, abort, kErrQ, status)) break;
        mbar_arrive_expect_tx(q_full, 2 * TR::Q_TILE_BYTES);
#pragma unroll
        for (int t = 0; t < 2; ++t)
#pragma unroll
          for (int c = 0; c < TR::NCH; ++c)
            tma_load_3d(smem_u32(smem + TR::OFF_Q + t * TR::Q_TILE_BYTES + c * TR::Q_CHUNK_BYTES),
                        &tmQ, c * TR::CHUNK, w.head, w.g.q_start + w.q0 + t * BM, q_full);
        for (int j = 0; j < w.nmax; ++j, ++kv_it) {
          const int s = kv_it % ST, ph = (kv_it / ST) & 1;
          int row = w.g.k_start + j * BN, page = 0;
          if (p.block_table != nullptr) {  // paged: the tile lies inside one page
            page = p.block_table[int64_t(w.seq) * p.max_pages + (j * BN) / p.page_size];
            row = (j * BN) % p.page_size;
          }
          if (kv_it >= ST && !mbar_wait(k_empty(s), ph ^ 1, abort, kErrKEmpty, status)) { ok = false; break; }
          if (kv_it != p.debug_withhold_kv) {
            mbar_arrive_expect_tx(k_full(s), TR::KV_BYTES);
#pragma unroll
            for (int c = 0; c < TR::NCH; ++c) {
              const uint32_t dst = smem_u32(smem + TR::OFF_K + s * TR::KV_BYTES + c * TR::KV_CHUNK_BYTES);
              if (p.block_table != nullptr)
                tma_load_4d_hint(dst, &tmK, c * TR::CHUNK, w.kvh, row, page, k_full(s), pol_kv);
              else
                tma_load_3d_hint(dst, &tmK, c * TR::CHUNK, w.kvh, row, k_full(s), pol_kv);
            }
            last_k[s] = kv_it;
          }
          if (kv_it >= ST && !mbar_wait(v_empty(s), ph ^ 1, abort, kErrVEmpty, status)) { ok = false; break; }
          mbar_arrive_expect_tx(v_full(s), TR::KV_BYTES);
#pragma unroll
          for (int c = 0; c < TR::NCH; ++c) {
            const uint32_t dst = smem_u32(smem + TR::OFF_V + s * TR::KV_BYTES + c * TR::KV_CHUNK_BYTES);
            if (p.block_table != nullptr)
              tma_load_4d_hint(dst, &tmV, c * TR::CHUNK, w.kvh, row, page, v_full(s), pol_kv);
            else
              tma_load_3d_hint(dst, &tmV, c * TR::CHUNK, w.kvh, row, v_full(s), pol_kv);
          }
          last_v[s] = kv_it;
        }
        ++tile_it;
      }
      // every copy this thread issued has landed before it leaves its role (on the
      // normal path the consumers already waited for them, so this returns at once)
      if (tile_it > 0) mbar_wait_drain(q_full, (tile_it - 1) & 1, kErrDrain, status);
      for (int s = 0; s < ST; ++s) {
        if (last_k[s] >= 0) mbar_wait_drain(k_full(s), (last_k[s] / ST) & 1, kErrDrain, status);
        if (last_v[s] >= 0) mbar_wait_drain(v_full(s), (last_v[s] / ST) & 1, kErrDrain, status);
      }
    }
   } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const int fmt = TR::FP8 ? 0 : p.in_fmt;
      const uint32_t idesc_qk = make_idesc(BM, BN, fmt, fmt, 0, 0);
      const uint32_t idesc_pv = make_idesc(BM, D, fmt, fmt, 0, 1);
      auto issue_s = [&](int t, int stage) {
        const uint32_t sQ = smem_u32(smem + TR::OFF_Q + t * TR::Q_TILE_BYTES);
        const uint32_t sK = smem_u32(smem + TR::OFF_K + stage * TR::KV_BYTES);
#pragma unroll
        for (int kk = 0; kk < D / TR::MMA_K; ++kk) {
          const int off = kk * 32;  // bytes along D of this K-step
          const uint32_t ca = (off / 128) * TR::Q_CHUNK_BYTES + (off % 128);
          const uint32_t cb = (off / 128) * TR::KV_CHUNK_BYTES + (off % 128);
          const uint64_t adesc = make_desc_sw128(sQ + ca, 16, 1024);
          const uint64_t bdesc = make_desc_sw128(sK + cb, 16, 1024);
          if constexpr (TR::FP8)
            mma_f8_ss(tmem + uint32_t(TR::tm_s(t)), adesc, bdesc, idesc_qk, kk > 0 ? 1u : 0u);
          else
            mma_f16_ss(tmem + uint32_t(TR::tm_s(t)), adesc, bdesc, idesc_qk, kk > 0 ? 1u : 0u);
        }
        tc_commit(s_full(t));
      };
      // PV of one key slice (the caller has waited for that slice of P)
      auto issue_pv_slice = [&](int t, int stage, bool first, int h) {
        const uint32_t sV = smem_u32(smem + TR::OFF_V + stage * TR::KV_BYTES);
        constexpr int KS = BN / TR::MMA_K / TR::P_SPLIT;  // K-steps per slice
#pragma unroll
        for (int k2 = 0; k2 < KS; ++k2) {
          const int kk = h * KS + k2;
          const uint64_t bdesc = make_desc_sw128(sV + kk * TR::MMA_K * 128, TR::KV_CHUNK_BYTES, 1024);
          const uint32_t a_tmem = tmem + uint32_t(TR::tm_s(t) + kk * 8);
          const uint32_t acc = (!first || kk > 0) ? 1u : 0u;
          if constexpr (TR::FP8)
            mma_f8_ts(tmem + uint32_t(TR::tm_o(t)), a_tmem, bdesc, idesc_pv, acc);
          else
            mma_f16_ts(tmem + uint32_t(TR::tm_o(t)), a_tmem, bdesc, idesc_pv, acc);
        }
      };
      // e4m3 split tile: the second PV term, lo = P - hi, from the next 32 TMEM columns
      auto issue_pv_lo = [&](int t, int stage) {
        const uint32_t sV = smem_u32(smem + TR::OFF_V + stage * TR::KV_BYTES);
#pragma unroll
        for (int kk = 0; kk < BN / TR::MMA_K; ++kk) {
          const uint64_t bdesc = make_desc_sw128(sV + kk * TR::MMA_K * 128, TR::KV_CHUNK_BYTES, 1024);
          mma_f8_ts(tmem + uint32_t(TR::tm_o(t)), tmem + uint32_t(TR::tm_s(t) + 32 + kk * 8), bdesc,
                    idesc_pv, 1u);
        }
      };
      int kv_it = 0, tile_it = 0;
      int p_cnt[2] = {0, 0};          // P hand-offs consumed per query tile (p_full phases)
      int ofree_cnt[2] = {0, 0};      // epilogues that read O_t (o_free phases) ...
      int ofree_seen[2] = {0, 0};     // ... and how many of them this thread has waited for
      bool ok = true;
      for (int it_tile = 0, tile = snake_tile(0); (TR::PERSISTENT || it_tile == 0) && ok && tile < n_tiles; tile = snake_tile(++it_tile)) {
        TileWork w;
        if (!tile_work(p, tile, BN, w)) continue;
        if (!mbar_wait(q_full, tile_it & 1, abort, kErrQ, status)) { ok = false; break; }
        tc_fence_after();
        if (w.nmax > 0) {
          const int s0 = kv_it % ST;
          if (!mbar_wait(k_full(s0), (kv_it / ST) & 1, abort, kErrKFull, status)) { ok = false; break; }
          tc_fence_after();
          if (w.n_t[0] > 0) issue_s(0, s0);
          if (w.n_t[1] > 0) issue_s(1, s0);
          tc_commit(k_empty(s0));
        }
        for (int j = 0; ok && j < w.nmax; ++j) {
          const int it = kv_it + j, s = it % ST;
          bool v_ready = false, k_next_ready = false;
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            if (j >= w.n_t[t]) continue;
            if (j == 0 && ofree_seen[t] < ofree_cnt[t]) {
              // PV_t(0) overwrites O_t: the previous tile's epilogue must have read it
              if (!mbar_wait(o_free(t), ofree_seen[t] & 1, abort, kErrODone, status)) { ok = false; break; }
              ++ofree_seen[t];
            }
            if (!v_ready) {
              if (!mbar_wait(v_full(s), (it / ST) & 1, abort, kErrVFull, status)) { ok = false; break; }
              v_ready = true;
            }
#pragma unroll
            for (int h = 0; h < TR::P_SPLIT; ++h) {
              if (!mbar_wait(p_full(t, h), p_cnt[t] & 1, abort, kErrPFull, status)) { ok = false; break; }
              tc_fence_after();
              issue_pv_slice(t, s, j == 0, h);
            }
            if (!ok) break;
            if constexpr (TR::FP8) {
              if (j == 0 && fp8_split_first(p, w, t)) issue_pv_lo(t, s);
            }
            ++p_cnt[t];
            tc_commit(o_done(t));
            if (j + 1 < w.n_t[t]) {
              const int s1 = (it + 1) % ST;
              if (!k_next_ready) {
                if (!mbar_wait(k_full(s1), ((it + 1) / ST) & 1, abort, kErrKFull, status)) {
                  ok = false;
                  break;
                }
                k_next_ready = true;
                tc_fence_after();
              }
              issue_s(t, s1);
            }
          }
          if (!ok) break;
          tc_commit(v_empty(s));
          if (k_next_ready) tc_commit(k_empty((it + 1) % ST));
        }
        if (!ok) break;
        // every S MMA of this tile is issued: its Q buffers are free once they complete
        tc_commit(q_empty);
        for (int t = 0; t < 2; ++t)
          if (w.n_t[t] > 0) ++ofree_cnt[t];
        kv_it += w.nmax;
        ++tile_it;
      }
      // every MMA issued above has completed before TMEM is released
      tc_commit(td_bar);
      mbar_wait_drain(td_bar, 0, kErrDrain, status);
    }
   }
  } else {
    setmaxnreg_inc<TR::REGS_SOFTMAX>();
    // ------------------------------------------------------------ softmax + epilogue
    const int t = warp >> 2;  // query tile slot of this warpgroup
    const int wq = warp & 3;
    const int r = wq * 32 + lane;
    const uint32_t t_lane = tmem + (uint32_t(wq * 32) << 16);
    int s_cnt = 0;   // S_t completions consumed (s_full phases)
    int pv_cnt = 0;  // PV_t MMAs issued for this slot so far (o_done phases)
    bool aborted = false;

    for (int it_tile = 0, tile = snake_tile(0); (TR::PERSISTENT || it_tile == 0) && !aborted && tile < n_tiles; tile = snake_tile(++it_tile)) {
      TileWork w;
      if (!tile_work(p, tile, BN, w)) continue;
      if (w.rows_t[t] <= 0) continue;  // this query tile lies past the sequence end
      const int first = w.q0 + t * BM;
      const int key_lim = first + r + w.diag;
      const int n = w.n_t[t];
      float scale = p.scale_log2;
      float vscale = 1.0f;
      if (p.q_descale) scale *= p.q_descale[w.kvh];
      if (p.k_descale) scale *= p.k_descale[w.kvh];
      if (p.v_descale) vscale = p.v_descale[w.kvh];
      const uint64_t scale2 = f2pack(scale, scale);
      float m = kNegInf, l = 0.f;

      // one K/V tile of the online softmax (SPLIT: its e4m3 P as two terms, fp8_p_to_tmem);
      // false when a bounded wait gave up
      auto softmax_tile = [&](int j, auto split_tag) -> bool {
        constexpr bool SPLIT = decltype(split_tag)::value;
        bool ok = mbar_wait(s_full(t), s_cnt & 1, abort, kErrSFull, status);
        if (!__all_sync(0xffffffffu, ok)) return false;
        ++s_cnt;
        tc_fence_after();
        uint32_t sr[BN / 32][32];
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) tmem_ld32(t_lane + uint32_t(TR::tm_s(t) + c * 32), sr[c]);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) reg_fence32(sr[c]);

        const int kbase = j * BN;
        const bool need_mask =
            (kbase + BN > w.g.k_len) || (p.causal && kbase + BN - 1 > first + w.diag);
        if (need_mask) {
#pragma unroll
          for (int c = 0; c < BN / 32; ++c)
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              const int key = kbase + c * 32 + e;
              if (key >= w.g.k_len || (p.causal && key > key_lim)) sr[c][e] = __float_as_uint(kNegInf);
            }
        }
        float mx4[4] = {kNegInf, kNegInf, kNegInf, kNegInf};
#pragma unroll
        for (int c = 0; c < BN / 32; ++c)
#pragma unroll
          for (int e = 0; e < 32; e += 2)
            mx4[c] = fmax3(mx4[c], __uint_as_float(sr[c][e]), __uint_as_float(sr[c][e + 1]));
        const float mx = fmax3(fmaxf(mx4[0], mx4[1]), mx4[2], mx4[3]);
        const float m_new = fmaxf(m, mx);
        if (j == 0) {
          m = m_new;
        } else {
          const bool need = (m_new - m) * scale > kRescaleThreshold;
          if (__any_sync(0xffffffffu, need)) {
            // PV_t(j-1) is complete: S_t(j) was issued after it and has completed.
            const float f = need ? ex2_approx((m - m_new) * scale) : 1.0f;
            if (need) { l *= f; m = m_new; }
            const uint64_t f2 = f2pack(f, f);
#pragma unroll 1
            for (int c = 0; c < D / 32; ++c) {
              uint32_t o[32];
              tmem_ld32(t_lane + uint32_t(TR::tm_o(t) + c * 32), o);
              tmem_wait_ld();
              reg_fence32(o);
#pragma unroll
              for (int e = 0; e < 32; e += 2) {
                const uint64_t v = fmul2(f2pack(__uint_as_float(o[e]), __uint_as_float(o[e + 1])), f2);
                o[e] = __float_as_uint(f2lo(v));
                o[e + 1] = __float_as_uint(f2hi(v));
              }
              tmem_st32(t_lane + uint32_t(TR::tm_o(t) + c * 32), o);
            }
            tmem_wait_st();
          }
        }
        const float neg_m = (m == kNegInf) ? 0.f : -m * scale;
        const uint64_t negm2 = f2pack(neg_m, neg_m);
        uint64_t rs2[2] = {0ull, 0ull};
        if constexpr (TR::FP8) {
          rs2[0] = fp8_p_to_tmem<TR, SPLIT>(sr, scale2, negm2, t_lane + uint32_t(TR::tm_s(t)));
          tmem_wait_st();
          tc_fence_before();
#pragma unroll
          for (int h = 0; h < TR::P_SPLIT; ++h) mbar_arrive(p_full(t, h));
        } else {
          // P in 64-key halves: exps of a half are kept (as fp32 bits, in place of S) for
          // the row sum, which is added up after P has been handed to the MMA warp
          static_assert(TR::FP8 || BN / 64 == 2, "bf16 path assumes two 64-key halves");
#pragma unroll
          for (int half = 0; half < BN / 64; ++half) {
            uint32_t pw[32];
#pragma unroll
            for (int e = 0; e < 64; e += 2) {
              const int c = half * 2 + (e >> 5), ee = e & 31;
              const uint64_t a = ffma2(f2pack(__uint_as_float(sr[c][ee]), __uint_as_float(sr[c][ee + 1])), scale2, negm2);
              const uint64_t ex = exp2_pair<TR>(half * 32 + (e >> 1), a);
              const float x0 = f2lo(ex), x1 = f2hi(ex);
              sr[c][ee] = __float_as_uint(x0);
              sr[c][ee + 1] = __float_as_uint(x1);
              pw[e >> 1] = p.in_fmt ? pack_bf16x2(x0, x1) : pack_f16x2(x0, x1);
            }
            tmem_st32(t_lane + uint32_t(TR::tm_s(t) + half * 32), pw);
            if (TR::P_SPLIT == 2 || half == BN / 64 - 1) {
              tmem_wait_st();
              tc_fence_before();
              if (TR::P_SPLIT == 2) {
                mbar_arrive(p_full(t, half));
              } else {
#pragma unroll
                for (int h = 0; h < TR::P_SPLIT; ++h) mbar_arrive(p_full(t, h));
              }
            }
          }
#pragma unroll
          for (int c = 0; c < BN / 32; ++c)
#pragma unroll
            for (int e = 0; e < 32; e += 4) {
              rs2[0] = fadd2(rs2[0], f2pack(__uint_as_float(sr[c][e]), __uint_as_float(sr[c][e + 1])));
              rs2[1] = fadd2(rs2[1], f2pack(__uint_as_float(sr[c][e + 2]), __uint_as_float(sr[c][e + 3])));
            }
        }
        const uint64_t rs = fadd2(rs2[0], rs2[1]);
        l += f2lo(rs) + f2hi(rs);
        return true;
      };
      // e4m3: the first tile may be split (fp8_split_first); it runs before the loop, so
      // that the loop holds one copy of the step
      int j0 = 0;
      if constexpr (TR::FP8) {
        if (n > 0 && fp8_split_first(p, w, t)) {
          if (!softmax_tile(0, std::true_type{})) aborted = true;
          j0 = 1;
        }
      }
      for (int j = j0; !aborted && j < n; ++j) {
        if (!softmax_tile(j, std::false_type{})) aborted = true;
      }
      if (aborted) break;

      // ---------------------------------------------------------- epilogue of this tile
      if (n > 0) {
        // the last PV_t of this tile; PV_t of the next tile waits for o_free below
        pv_cnt += n;
        bool ok = mbar_wait(o_done(t), (pv_cnt - 1) & 1, abort, kErrODone, status);
        if (!__all_sync(0xffffffffu, ok)) { aborted = true; break; }
        tc_fence_after();
      }
      const bool valid = r < w.rows_t[t];
      const int64_t grow = int64_t(w.g.q_start) + first + r;
      // a row that saw no key has m = -inf (the emulated exp2 maps -inf to ~1e-38, not 0,
      // so l alone cannot tell)
      const bool any_key = (m != kNegInf) && (l > 0.f);
      const float lse_new = any_key ? (m * scale + lg2_approx(l)) * kLn2 : kNegInf;
      float* lse_ptr = p.lse + grow * p.Hq + w.head;
      float ca = 0.f, cb = any_key ? vscale / l : 0.f, lse_out = lse_new;
      bool write = valid;
      bool read_acc = false;
      if (valid && p.accumulate) {
        const float acc_lse = *lse_ptr;
        if (lse_new == kNegInf) {
          write = false;
        } else if (acc_lse != kNegInf) {
          const float mm = fmaxf(acc_lse, lse_new);
          const float wa = ex2_approx((acc_lse - mm) * kLog2e);
          const float wb = ex2_approx((lse_new - mm) * kLog2e);
          const float inv = 1.0f / (wa + wb);
          ca = wa * inv;
          cb *= wb * inv;
          lse_out = mm + lg2_approx(wa + wb) * kLn2;
          read_acc = true;
        }
      }
      uint8_t* orow = static_cast<uint8_t*>(p.out) + (grow * p.Hq + w.head) * int64_t(D) * 2;
      const bool has_o = n > 0;  // warpgroup-uniform
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        if (has_o) {
          tmem_ld32(t_lane + uint32_t(TR::tm_o(t) + c * 32), o);
          tmem_wait_ld();
          reg_fence32(o);
          if (c == D / 32 - 1) {
            // all of O_t has been read: the next tile's PV_t may overwrite it
            tc_fence_before();
            mbar_arrive(o_free(t));
          }
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = 0u;
        }
        if (write) {
          uint4* dst = reinterpret_cast<uint4*>(orow + c * 64);
          float f[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) f[e] = has_o ? __uint_as_float(o[e]) * cb : 0.f;
          if (read_acc) {
#pragma unroll
            for (int v4 = 0; v4 < 4; ++v4) {
              const uint4 a = dst[v4];
              const uint32_t wd[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                float lo, hi;
                if (p.out_bf16) {
                  lo = __uint_as_float(wd[i] << 16);
                  hi = __uint_as_float(wd[i] & 0xFFFF0000u);
                } else {
                  const float2 tt = __half22float2(*reinterpret_cast<const __half2*>(&wd[i]));
                  lo = tt.x; hi = tt.y;
                }
                f[v4 * 8 + 2 * i] = fmaf(lo, ca, f[v4 * 8 + 2 * i]);
                f[v4 * 8 + 2 * i + 1] = fmaf(hi, ca, f[v4 * 8 + 2 * i + 1]);
              }
            }
          }
#pragma unroll
          for (int v4 = 0; v4 < 4; ++v4) {
            uint32_t wd[4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
              wd[i] = p.out_bf16 ? pack_bf16x2(f[v4 * 8 + 2 * i], f[v4 * 8 + 2 * i + 1])
                                 : pack_f16x2(f[v4 * 8 + 2 * i], f[v4 * 8 + 2 * i + 1]);
            dst[v4] = make_uint4(wd[0], wd[1], wd[2], wd[3]);
          }
        }
      }
      if (write) *lse_ptr = lse_out;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 9) tmem_dealloc(tmem, TR::TM_COLS);
}

#include "ring_fused.cuh"

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

// 3-D view [rows, heads, D] with a 128-byte-swizzled box of (128 bytes, 1 head, box_rows).
int make_map(CUtensorMap* map, const void* base, int64_t rows, int heads, int D, int elem,
             int box_rows) {
  EncodeTiledFn enc = get_encode_fn();
  FA4CP_CHECK_ARG(enc != nullptr, "cuTensorMapEncodeTiled is unavailable");
  const cuuint64_t dims[3] = {cuuint64_t(D), cuuint64_t(heads), cuuint64_t(rows)};
  const cuuint64_t strides[2] = {cuuint64_t(D) * elem, cuuint64_t(heads) * D * elem};
  const cuuint32_t box[3] = {cuuint32_t(128 / elem), 1, cuuint32_t(box_rows)};
  const cuuint32_t es[3] = {1, 1, 1};
  CUresult r = enc(map, elem == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_UINT16,
                   3, const_cast<void*>(base), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_last_error("cuTensorMapEncodeTiled failed (%d)", int(r));
    return FA4CP_ERR_CUDA;
  }
  return FA4CP_OK;
}

// Opt a kernel into its dynamic shared memory once per device (the attribute is per device;
// one bit per device id for up to 64 devices, set after the call succeeded).
template <class Fn>
int smem_optin(Fn kernel, int bytes, std::atomic<uint64_t>& done) {
  int dev = 0;
  FA4CP_CHECK_CUDA(cudaGetDevice(&dev));
  const uint64_t bit = dev < 64 ? (uint64_t(1) << dev) : 0;
  if (bit != 0 && (done.load() & bit)) return FA4CP_OK;
  FA4CP_CHECK_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  done.fetch_or(bit);
  return FA4CP_OK;
}

template <class TR>
int launch(const void* q, const void* k, const void* v, int64_t total_q, int64_t total_k,
           int max_seqlen_q, const Params& p0, cudaStream_t stream) {
  static std::atomic<uint64_t> optin{0};
  if (int rc0 = smem_optin(attn_fwd_kernel<TR>, TR::SMEM_BYTES, optin)) return rc0;
  CUtensorMap mq, mk, mv;
  int rc = make_map(&mq, q, total_q, p0.Hq, TR::D, TR::ELEM, BM);
  if (rc) return rc;
  if (total_k > 0) {
    if ((rc = make_map(&mk, k, total_k, p0.Hkv, TR::D, TR::ELEM, TR::BN))) return rc;
    if ((rc = make_map(&mv, v, total_k, p0.Hkv, TR::D, TR::ELEM, TR::BN))) return rc;
  } else {  // no keys anywhere: the kernel never loads K/V; any valid map will do
    mk = mq;
    mv = mq;
  }
  Params p = p0;
  p.n_qtiles = (max_seqlen_q + BM - 1) / BM;
  if (p.n_qtiles <= 0) return FA4CP_OK;
  FA4CP_CHECK_ARG(int64_t(p.n_qtiles + kQtileChunk) * p.Hq < (int64_t(1) << 31) && p.nseq <= 65535,
                  "grid too large");
  dim3 grid(cta_grid_x(p.n_qtiles, p.Hq), 1u, unsigned(p.nseq));
  attn_fwd_kernel<TR><<<grid, kThreads, TR::SMEM_BYTES, stream>>>(mq, mk, mv, p);
  return check_launch("attn_fwd");
}

template <class TR>
int launch2(const void* q, const void* k, const void* v, int64_t total_q, int64_t total_k,
            int max_seqlen_q, const Params& p0, cudaStream_t stream) {
  static std::atomic<uint64_t> optin{0};
  if (int rc0 = smem_optin(attn_fwd_2q_kernel<TR>, TR::SMEM_BYTES, optin)) return rc0;
  CUtensorMap mq, mk, mv;
  int rc = make_map(&mq, q, total_q, p0.Hq, TR::D, TR::ELEM, BM);
  if (rc) return rc;
  if (total_k > 0) {
    if ((rc = make_map(&mk, k, total_k, p0.Hkv, TR::D, TR::ELEM, TR::BN))) return rc;
    if ((rc = make_map(&mv, v, total_k, p0.Hkv, TR::D, TR::ELEM, TR::BN))) return rc;
  } else {
    mk = mq;
    mv = mq;
  }
  Params p = p0;
  p.n_qtiles = (max_seqlen_q + 2 * BM - 1) / (2 * BM);
  if (p.n_qtiles <= 0) return FA4CP_OK;
  FA4CP_CHECK_ARG(int64_t(p.n_qtiles + kQtileChunk) * p.Hq * p.nseq < (int64_t(1) << 31),
                  "too many tiles");
  p.n_tiles = persistent_tiles(p.n_qtiles, p.Hq, p.nseq);
  // persistent: one CTA per SM, each walking the tile schedule with a stride of the grid
  static int sms = 0;
  if (sms == 0) {
    int dev = 0;
    FA4CP_CHECK_CUDA(cudaGetDevice(&dev));
    FA4CP_CHECK_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  }
  const int ctas = sms - (t_sm_reserve < sms / 2 ? t_sm_reserve : sms / 2);
  const int grid = (TR::PERSISTENT && p.n_tiles > ctas) ? ctas : p.n_tiles;
  attn_fwd_2q_kernel<TR><<<grid, TR::THREADS, TR::SMEM_BYTES, stream>>>(mq, mk, mv, p);
  return check_launch("attn_fwd_2q");
}

bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

// 4-D view [slots, rows, heads, D] (slot stride in bytes) with a box of (128 bytes, 1 head,
// box_rows, 1 slot): the receive slots of the ring, one per hop.
int make_map4(CUtensorMap* map, const void* base, int64_t rows, int heads, int D, int elem,
              int box_rows, int slots, int64_t slot_stride) {
  EncodeTiledFn enc = get_encode_fn();
  FA4CP_CHECK_ARG(enc != nullptr, "cuTensorMapEncodeTiled is unavailable");
  const cuuint64_t dims[4] = {cuuint64_t(D), cuuint64_t(heads), cuuint64_t(rows), cuuint64_t(slots)};
  const cuuint64_t strides[3] = {cuuint64_t(D) * elem, cuuint64_t(heads) * D * elem,
                                 cuuint64_t(slot_stride)};
  const cuuint32_t box[4] = {cuuint32_t(128 / elem), 1, cuuint32_t(box_rows), 1};
  const cuuint32_t es[4] = {1, 1, 1, 1};
  CUresult r = enc(map, elem == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_UINT16,
                   4, const_cast<void*>(base), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_last_error("cuTensorMapEncodeTiled (4-D) failed (%d)", int(r));
    return FA4CP_ERR_CUDA;
  }
  return FA4CP_OK;
}

// Paged K/V through the two-tile kernel: the pools [num_pages, page_size, Hkv, D] are 4-D
// tensor maps (page = the slowest coordinate); the producer looks up each K/V tile's page.
template <class TR>
int launch2_paged(const void* q, const void* k_pages, const void* v_pages, int num_pages,
                  int64_t total_q, int max_seqlen_q, const Params& p0, cudaStream_t stream) {
  static std::atomic<uint64_t> optin{0};
  if (int rc0 = smem_optin(attn_fwd_2q_kernel<TR>, TR::SMEM_BYTES, optin)) return rc0;
  FA4CP_CHECK_ARG(p0.page_size % TR::BN == 0, "page_size %d must be a multiple of %d",
                  p0.page_size, TR::BN);
  CUtensorMap mq, mk, mv;
  int rc;
  if ((rc = make_map(&mq, q, total_q, p0.Hq, TR::D, TR::ELEM, BM))) return rc;
  const int64_t page_bytes = int64_t(p0.page_size) * p0.Hkv * TR::D * TR::ELEM;
  if ((rc = make_map4(&mk, k_pages, p0.page_size, p0.Hkv, TR::D, TR::ELEM, TR::BN, num_pages, page_bytes)))
    return rc;
  if ((rc = make_map4(&mv, v_pages, p0.page_size, p0.Hkv, TR::D, TR::ELEM, TR::BN, num_pages, page_bytes)))
    return rc;
  Params p = p0;
  p.n_qtiles = (max_seqlen_q + 2 * BM - 1) / (2 * BM);
  if (p.n_qtiles <= 0) return FA4CP_OK;
  FA4CP_CHECK_ARG(int64_t(p.n_qtiles + kQtileChunk) * p.Hq * p.nseq < (int64_t(1) << 31),
                  "too many tiles");
  p.n_tiles = persistent_tiles(p.n_qtiles, p.Hq, p.nseq);
  static int sms = 0;
  if (sms == 0) {
    int dev = 0;
    FA4CP_CHECK_CUDA(cudaGetDevice(&dev));
    FA4CP_CHECK_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  }
  const int grid = (TR::PERSISTENT && p.n_tiles > sms) ? sms : p.n_tiles;
  attn_fwd_2q_kernel<TR><<<grid, TR::THREADS, TR::SMEM_BYTES, stream>>>(mq, mk, mv, p);
  return check_launch("attn_fwd_2q (paged)");
}

template <class TR>
int launch_ring_fused(const void* q, const void* k, const void* v, const void* slots_k,
                      const void* slots_v, int64_t slot_stride, int64_t total, int max_seqlen,
                      const RingFusedParams& p0, cudaStream_t stream) {
  using KernelFn = void (*)(CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap,
                           RingFusedParams);
  KernelFn kernel, split_kernel = nullptr;
  if constexpr (TR::PERSISTENT) {
    kernel = ring_fused_persistent_kernel<TR, false>;
    if constexpr (TR::FP8) split_kernel = ring_fused_persistent_kernel<TR, true>;
  } else {
    kernel = ring_fused_kernel<TR>;
  }
  static std::atomic<uint64_t> optin{0}, optin_split{0};
  if (int rc0 = smem_optin(kernel, TR::SMEM_BYTES, optin)) return rc0;
  if (split_kernel != nullptr) {
    if (int rc0 = smem_optin(split_kernel, TR::SMEM_BYTES, optin_split)) return rc0;
  }
  RingFusedParams p = p0;
  p.n_pairs = (max_seqlen / 2 + 2 * BM - 1) / (2 * BM);
  if (p.n_pairs <= 0 || total <= 0) return FA4CP_OK;
  FA4CP_CHECK_ARG(int64_t(2) * ((p.n_pairs + kQtileChunk - 1) / kQtileChunk + 1) * kQtileChunk * p.Hq * p.nseq <
                      (int64_t(1) << 31), "too many tiles");
  p.n_tiles = int(ring_grid(p.n_pairs, p.Hq, p.nseq));
  CUtensorMap mq, mk0, mv0, mks, mvs;
  int rc;
  if ((rc = make_map(&mq, q, total, p.Hq, TR::D, TR::ELEM, BM))) return rc;
  if ((rc = make_map(&mk0, k, total, p.Hkv, TR::D, TR::ELEM, TR::BN))) return rc;
  if ((rc = make_map(&mv0, v, total, p.Hkv, TR::D, TR::ELEM, TR::BN))) return rc;
  if (p.S > 1) {
    if ((rc = make_map4(&mks, slots_k, total, p.Hkv, TR::D, TR::ELEM, TR::BN, p.S - 1, slot_stride)))
      return rc;
    if ((rc = make_map4(&mvs, slots_v, total, p.Hkv, TR::D, TR::ELEM, TR::BN, p.S - 1, slot_stride)))
      return rc;
  } else {
    mks = mk0;  // no step reads a slot
    mvs = mv0;
  }
  static int sms = 0;
  if (sms == 0) {
    int dev = 0;
    FA4CP_CHECK_CUDA(cudaGetDevice(&dev));
    FA4CP_CHECK_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  }
  // persistent (FP8): one CTA per SM walking the tile list; otherwise one CTA per tile
  const int grid = (TR::PERSISTENT && p.n_tiles > sms) ? sms : p.n_tiles;
  kernel<<<grid, TR::THREADS, TR::SMEM_BYTES, stream>>>(mq, mk0, mv0, mks, mvs, p);
  if (int rc = check_launch("ring_fused")) return rc;
  // e4m3: the CTA tiles with a short-keyed row (ring_split_all), P split in two terms.  With one
  // sequence the host knows whether any exists: the early-half pair 0 sees 1 + rank * h keys,
  // the late-half pair 0 h + 1 or more (h = half length); packed sequences always run the pass.
  // It holds few tiles (one pair per head for a long sequence), so a small grid walks the list.
  const int64_t hh = total / 2;
  const bool need_split = p.nseq > 1 || int64_t(p.rank) * hh + 1 < 128 || hh + 1 < 128;
  if (split_kernel != nullptr && need_split) {
    const int grid_split = p.n_tiles < 64 ? p.n_tiles : 64;
    split_kernel<<<grid_split, TR::THREADS, TR::SMEM_BYTES, stream>>>(mq, mk0, mv0, mks, mvs, p);
    return check_launch("ring_fused (split pass)");
  }
  return FA4CP_OK;
}

// The one-query-tile ring kernel (head_dim 256): one CTA per 128-row query tile of a half.
template <class TR>
int launch_ring_fused_1q(const void* q, const void* k, const void* v, const void* slots_k,
                         const void* slots_v, int64_t slot_stride, int64_t total, int max_seqlen,
                         const RingFusedParams& p0, cudaStream_t stream) {
  static std::atomic<uint64_t> optin{0};
  if (int rc0 = smem_optin(ring_fused_1q_kernel<TR>, TR::SMEM_BYTES, optin)) return rc0;
  RingFusedParams p = p0;
  p.n_pairs = (max_seqlen / 2 + BM - 1) / BM;  // query tiles per half
  if (p.n_pairs <= 0 || total <= 0) return FA4CP_OK;
  FA4CP_CHECK_ARG(int64_t(2) * ((p.n_pairs + kQtileChunk - 1) / kQtileChunk + 1) * kQtileChunk * p.Hq * p.nseq <
                      (int64_t(1) << 31), "too many tiles");
  p.n_tiles = int(ring_grid(p.n_pairs, p.Hq, p.nseq));
  CUtensorMap mq, mk0, mv0, mks, mvs;
  int rc;
  if ((rc = make_map(&mq, q, total, p.Hq, TR::D, TR::ELEM, BM))) return rc;
  if ((rc = make_map(&mk0, k, total, p.Hkv, TR::D, TR::ELEM, TR::BN))) return rc;
  if ((rc = make_map(&mv0, v, total, p.Hkv, TR::D, TR::ELEM, TR::BN))) return rc;
  if (p.S > 1) {
    if ((rc = make_map4(&mks, slots_k, total, p.Hkv, TR::D, TR::ELEM, TR::BN, p.S - 1, slot_stride)))
      return rc;
    if ((rc = make_map4(&mvs, slots_v, total, p.Hkv, TR::D, TR::ELEM, TR::BN, p.S - 1, slot_stride)))
      return rc;
  } else {
    mks = mk0;  // no step reads a slot
    mvs = mv0;
  }
  ring_fused_1q_kernel<TR><<<p.n_tiles, kThreads, TR::SMEM_BYTES, stream>>>(mq, mk0, mv0, mks, mvs, p);
  return check_launch("ring_fused_1q");
}

}  // namespace
}  // namespace fa4cp

using namespace fa4cp;

namespace fa4cp {
namespace {
// fa4cp_attn_fwd without its check that descales come with e4m3 operands only: the bf16 x
// e4m3-K/V path (fa4cp_attn_fwd_kv8) converts K/V to bf16 exactly and hands the descales to
// the kernel, which folds them into its fp32 score scale and output factor.
int attn_fwd_impl(const void* q, const void* k, const void* v, void* out, float* lse,
                  const int32_t* cu_q, const int32_t* cu_k, int32_t nseq, int32_t max_seqlen_q,
                  int64_t total_q, int64_t total_k, int32_t num_heads_q, int32_t num_heads_kv,
                  int32_t head_dim, int32_t in_dtype, int32_t out_dtype, int32_t pattern,
                  int32_t causal, float softmax_scale, const float* q_descale,
                  const float* k_descale, const float* v_descale, int32_t accumulate,
                  void* stream) {
  FA4CP_CHECK_ARG(nseq >= 1 && cu_q != nullptr, "cu_seqlens_q must describe >= 1 sequence");
  FA4CP_CHECK_ARG(pattern >= FA4CP_PATTERN_VARLEN && pattern <= FA4CP_PATTERN_BACK_Q,
                  "unknown pattern %d", pattern);
  FA4CP_CHECK_ARG(pattern != FA4CP_PATTERN_VARLEN || cu_k != nullptr, "cu_seqlens_k is required");
  FA4CP_CHECK_ARG(num_heads_q > 0 && num_heads_kv > 0 && num_heads_q % num_heads_kv == 0,
                  "H_q=%d not a multiple of H_kv=%d", num_heads_q, num_heads_kv);
  FA4CP_CHECK_ARG(total_q >= 0 && total_k >= 0 && max_seqlen_q >= 0, "bad sizes");
  FA4CP_CHECK_ARG(out_dtype == FA4CP_DTYPE_BF16 || out_dtype == FA4CP_DTYPE_F16,
                  "output dtype must be f16 or bf16");
  FA4CP_CHECK_ARG(softmax_scale > 0.f, "softmax_scale must be positive");
  const bool fp8 = in_dtype == FA4CP_DTYPE_E4M3;
  FA4CP_CHECK_ARG(fp8 || in_dtype == FA4CP_DTYPE_BF16 || in_dtype == FA4CP_DTYPE_F16,
                  "input dtype must be f16, bf16 or e4m3");
  if (total_q == 0) return FA4CP_OK;
  FA4CP_CHECK_ARG(q && out && lse && (total_k == 0 || (k && v)), "null tensor pointer");
  FA4CP_CHECK_ARG(aligned16(q) && aligned16(k) && aligned16(v) && aligned16(out),
                  "q/k/v/out must be 16-byte aligned");

  Params p{};
  p.cu_q = cu_q;
  p.cu_k = cu_k;
  p.out = out;
  p.lse = lse;
  p.q_descale = q_descale;
  p.k_descale = k_descale;
  p.v_descale = v_descale;
  p.nseq = nseq;
  p.Hq = num_heads_q;
  p.Hkv = num_heads_kv;
  p.group = num_heads_q / num_heads_kv;
  p.pattern = pattern;
  p.causal = causal ? 1 : 0;
  p.accumulate = accumulate ? 1 : 0;
  p.in_fmt = in_dtype == FA4CP_DTYPE_BF16 ? 1 : 0;
  p.out_bf16 = out_dtype == FA4CP_DTYPE_BF16 ? 1 : 0;
  p.scale_log2 = softmax_scale * kLog2e;
  p.debug_withhold_kv = -1;
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  if (fp8) {
    FA4CP_CHECK_ARG(out_dtype == FA4CP_DTYPE_BF16, "e4m3 inputs produce a bf16 output");
    if (head_dim == 128) return launch2<Traits2<128, 128, 3, true>>(q, k, v, total_q, total_k, max_seqlen_q, p, st);
  } else {
    if (head_dim == 128) return launch2<Traits2<128, 128, 2, false>>(q, k, v, total_q, total_k, max_seqlen_q, p, st);
    if (head_dim == 64) return launch2<Traits2<64, 128, 3, false>>(q, k, v, total_q, total_k, max_seqlen_q, p, st);
    // D=256: S (64 keys) x2 + O (256) fill 384 TMEM columns -- one query tile per CTA
    if (head_dim == 256) return launch<Traits<256, 64, 2, false>>(q, k, v, total_q, total_k, max_seqlen_q, p, st);
  }
  set_last_error("head_dim %d with dtype %d is not supported", head_dim, in_dtype);
  return FA4CP_ERR_UNSUPPORTED;
}
}  // namespace
}  // namespace fa4cp

extern "C" int fa4cp_attn_fwd(const void* q, const void* k, const void* v, void* out, float* lse,
                              const int32_t* cu_q, const int32_t* cu_k, int32_t nseq,
                              int32_t max_seqlen_q, int64_t total_q, int64_t total_k,
                              int32_t num_heads_q, int32_t num_heads_kv, int32_t head_dim,
                              int32_t in_dtype, int32_t out_dtype, int32_t pattern,
                              int32_t causal, float softmax_scale, const float* q_descale,
                              const float* k_descale, const float* v_descale, int32_t accumulate,
                              void* stream) {
  FA4CP_CHECK_ARG(in_dtype == FA4CP_DTYPE_E4M3 ||
                      (q_descale == nullptr && k_descale == nullptr && v_descale == nullptr),
                  "descales apply to e4m3 inputs only");
  return attn_fwd_impl(q, k, v, out, lse, cu_q, cu_k, nseq, max_seqlen_q, total_q, total_k,
                       num_heads_q, num_heads_kv, head_dim, in_dtype, out_dtype, pattern, causal,
                       softmax_scale, q_descale, k_descale, v_descale, accumulate, stream);
}

extern "C" int fa4cp_ring_attn_fused(const void* q, const void* k, const void* v,
                                     const void* slots_k, const void* slots_v,
                                     int64_t slot_stride, void* out, float* lse,
                                     const int32_t* cu, int32_t nseq, int32_t max_seqlen,
                                     int64_t total, int32_t num_heads_q, int32_t num_heads_kv,
                                     int32_t head_dim, int32_t dtype, float softmax_scale,
                                     const float* q_descale, const float* k_descales,
                                     const float* v_descales, int32_t nranks, int32_t rank,
                                     const uint32_t* arrived, uint32_t arrived_base,
                                     void* stream) {
  FA4CP_CHECK_ARG(dtype == FA4CP_DTYPE_E4M3 || (!q_descale && !k_descales && !v_descales),
                  "descales apply to e4m3 inputs only");
  return ring_attn_fused_flags(q, k, v, slots_k, slots_v, slot_stride, out, lse, cu, nseq,
                               max_seqlen, total, num_heads_q, num_heads_kv, head_dim, dtype,
                               softmax_scale, q_descale, k_descales, v_descales, nranks, rank,
                               arrived, arrived_base, 0, 1, 0, 0, stream);
}

extern "C" int fa4cp_ring_attn_fused_mixed(const void* q, const void* k, const void* v,
                                           const void* slots_k, const void* slots_v,
                                           int64_t slot_stride, void* out, float* lse,
                                           const int32_t* cu, int32_t nseq, int32_t max_seqlen,
                                           int64_t total, int32_t num_heads_q,
                                           int32_t num_heads_kv, int32_t head_dim,
                                           float softmax_scale, const float* k_descales,
                                           const float* v_descales, int32_t nranks, int32_t rank,
                                           const uint32_t* arrived, uint32_t arrived_base,
                                           void* stream) {
  FA4CP_CHECK_ARG(head_dim == 256, "the bf16 x e4m3-K/V ring kernel takes head_dim 256 (got %d)",
                  head_dim);
  return ring_attn_fused_flags(q, k, v, slots_k, slots_v, slot_stride, out, lse, cu, nseq,
                               max_seqlen, total, num_heads_q, num_heads_kv, head_dim,
                               FA4CP_DTYPE_BF16, softmax_scale, nullptr, k_descales, v_descales,
                               nranks, rank, arrived, arrived_base, 0, 1, 0, 0, stream);
}

extern "C" int fa4cp_ring_attn_fused_remote(const void* q, const void* k, const void* v,
                                            const void* slots_k, const void* slots_v,
                                            int64_t slot_stride, void* out, float* lse,
                                            const int32_t* cu, int32_t nseq, int32_t max_seqlen,
                                            int64_t total, int32_t num_heads_q,
                                            int32_t num_heads_kv, int32_t head_dim, int32_t dtype,
                                            float softmax_scale, int32_t nranks, int32_t rank,
                                            const uint32_t* arrived, uint32_t arrived_base,
                                            void* stream) {
  FA4CP_CHECK_ARG(dtype == FA4CP_DTYPE_BF16 || dtype == FA4CP_DTYPE_F16,
                  "the remote-only ring walk takes f16 / bf16");
  return ring_attn_fused_flags(q, k, v, slots_k, slots_v, slot_stride, out, lse, cu, nseq,
                               max_seqlen, total, num_heads_q, num_heads_kv, head_dim, dtype,
                               softmax_scale, nullptr, nullptr, nullptr, nranks, rank, arrived,
                               arrived_base, 0, 1, 1, 1, stream);
}

int fa4cp::ring_attn_fused_flags(const void* q, const void* k, const void* v,
                                 const void* slots_k, const void* slots_v, int64_t slot_stride,
                                 void* out, float* lse, const int32_t* cu, int32_t nseq,
                                 int32_t max_seqlen, int64_t total, int32_t num_heads_q,
                                 int32_t num_heads_kv, int32_t head_dim, int32_t dtype,
                                 float softmax_scale, const float* q_descale,
                                 const float* k_descales, const float* v_descales, int32_t nranks,
                                 int32_t rank, const uint32_t* arrived, uint32_t arrived_base,
                                 int32_t arrived_stride, int32_t arrived_step, int32_t first_step,
                                 int32_t accumulate, void* stream) {
  FA4CP_CHECK_ARG(arrived_stride >= 0 && arrived_step >= 0, "bad arrival flag layout");
  FA4CP_CHECK_ARG((first_step == 0 || first_step == 1) && (accumulate == 0 || accumulate == 1),
                  "bad first_step / accumulate");
  FA4CP_CHECK_ARG(first_step == 0 || dtype != FA4CP_DTYPE_E4M3,
                  "the remote-only walk is for f16 / bf16");
  FA4CP_CHECK_ARG(nseq >= 1 && cu != nullptr, "cu_seqlens must describe >= 1 sequence");
  FA4CP_CHECK_ARG(nranks >= 1 && nranks <= 64 && rank >= 0 && rank < nranks,
                  "bad ring size %d / rank %d", nranks, rank);
  FA4CP_CHECK_ARG(num_heads_q > 0 && num_heads_kv > 0 && num_heads_q % num_heads_kv == 0,
                  "H_q=%d not a multiple of H_kv=%d", num_heads_q, num_heads_kv);
  FA4CP_CHECK_ARG(total >= 0 && max_seqlen >= 0, "bad sizes");
  FA4CP_CHECK_ARG(softmax_scale > 0.f, "softmax_scale must be positive");
  const bool fp8 = dtype == FA4CP_DTYPE_E4M3;
  if (dtype != FA4CP_DTYPE_BF16 && dtype != FA4CP_DTYPE_F16 && !(fp8 && head_dim == 128)) {
    set_last_error("the ring kernel takes f16 / bf16 (D 64, 128, 256) or e4m3 (D 128); got dtype %d, D %d",
                   dtype, head_dim);
    return FA4CP_ERR_UNSUPPORTED;
  }
  // f16 / bf16 with descales: K/V are exact images of e4m3 values (the head_dim 256 kernel)
  FA4CP_CHECK_ARG(fp8 || head_dim == 256 || (!q_descale && !k_descales && !v_descales),
                  "descales apply to e4m3 inputs (or e4m3 K/V images at head_dim 256) only");
  FA4CP_CHECK_ARG(head_dim != 256 || (first_step == 0 && accumulate == 0),
                  "the head_dim 256 ring kernel walks every step in one launch");
  if (total == 0) return FA4CP_OK;
  FA4CP_CHECK_ARG(q && k && v && out && lse, "null tensor pointer");
  FA4CP_CHECK_ARG(nranks == 1 || (slots_k && slots_v), "slots are required for nranks > 1");
  FA4CP_CHECK_ARG(aligned16(q) && aligned16(k) && aligned16(v) && aligned16(out) &&
                      aligned16(slots_k) && aligned16(slots_v) && slot_stride % 16 == 0,
                  "tensors, slots and the slot stride must be 16-byte aligned");
  FA4CP_CHECK_ARG(nranks == 1 || slot_stride >= total * num_heads_kv * int64_t(head_dim) * (fp8 ? 1 : 2),
                  "slot stride smaller than one K/V shard");
  RingFusedParams p{};
  p.cu = cu;
  p.out = out;
  p.lse = lse;
  p.arrived = arrived;
  p.arrived_base = arrived_base;
  p.arrived_stride = arrived_stride;
  p.arrived_step = arrived_step;
  p.first_step = first_step;
  p.accumulate = accumulate;
  p.nseq = nseq;
  p.Hq = num_heads_q;
  p.Hkv = num_heads_kv;
  p.group = num_heads_q / num_heads_kv;
  p.S = nranks;
  p.rank = rank;
  p.in_fmt = dtype == FA4CP_DTYPE_BF16 ? 1 : 0;
  p.out_bf16 = (dtype == FA4CP_DTYPE_BF16 || fp8) ? 1 : 0;
  p.scale_log2 = softmax_scale * kLog2e;
  p.q_descale = q_descale;
  p.k_descales = k_descales;
  p.v_descales = v_descales;
  p.arrive_wait_ns = static_cast<unsigned long long>(g_ring_wait_ms.load()) * 1000000ull;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (fp8)  // persistent, as the per-step e4m3 kernel
    return launch_ring_fused<Traits2<128, 128, 3, true>>(q, k, v, slots_k, slots_v, slot_stride,
                                                         total, max_seqlen, p, st);
  if (head_dim == 128)
    return launch_ring_fused<Traits2<128, 128, 2, false>>(q, k, v, slots_k, slots_v, slot_stride,
                                                          total, max_seqlen, p, st);
  if (head_dim == 64)
    return launch_ring_fused<Traits2<64, 128, 3, false>>(q, k, v, slots_k, slots_v, slot_stride,
                                                         total, max_seqlen, p, st);
  if (head_dim == 256)
    return launch_ring_fused_1q<Traits<256, 64, 2, false>>(q, k, v, slots_k, slots_v,
                                                           slot_stride, total, max_seqlen, p, st);
  set_last_error("the ring kernel takes head_dim 64, 128 or 256 (got %d)", head_dim);
  return FA4CP_ERR_UNSUPPORTED;
}

extern "C" int fa4cp_ring_set_wait_timeout_ms(int32_t ms) {
  FA4CP_CHECK_ARG(ms >= 1 && ms <= 600000, "timeout %d ms not in [1, 600000]", ms);
  g_ring_wait_ms.store(ms);
  return FA4CP_OK;
}

extern "C" int fa4cp_attn_fwd_paged(const void* q, const void* k_pages, const void* v_pages,
                                    const int32_t* block_table, int32_t page_size,
                                    int32_t num_pages, int32_t max_pages_per_seq, void* out,
                                    float* lse, const int32_t* cu_q, const int32_t* cu_k,
                                    int32_t nseq, int32_t max_seqlen_q, int64_t total_q,
                                    int32_t num_heads_q, int32_t num_heads_kv, int32_t head_dim,
                                    int32_t in_dtype, int32_t out_dtype, int32_t causal,
                                    float softmax_scale, const float* q_descale,
                                    const float* k_descale, const float* v_descale,
                                    void* stream) {
  FA4CP_CHECK_ARG(nseq >= 1 && cu_q != nullptr && cu_k != nullptr,
                  "cu_seqlens_q/k must describe >= 1 sequence");
  FA4CP_CHECK_ARG(block_table != nullptr && page_size > 0 && num_pages > 0 && max_pages_per_seq > 0,
                  "paged K/V needs a block table, a page size and the pool size");
  FA4CP_CHECK_ARG(num_heads_q > 0 && num_heads_kv > 0 && num_heads_q % num_heads_kv == 0,
                  "H_q=%d not a multiple of H_kv=%d", num_heads_q, num_heads_kv);
  FA4CP_CHECK_ARG(total_q >= 0 && max_seqlen_q >= 0, "bad sizes");
  FA4CP_CHECK_ARG(out_dtype == FA4CP_DTYPE_BF16 || out_dtype == FA4CP_DTYPE_F16,
                  "output dtype must be f16 or bf16");
  FA4CP_CHECK_ARG(softmax_scale > 0.f, "softmax_scale must be positive");
  const bool fp8 = in_dtype == FA4CP_DTYPE_E4M3;
  FA4CP_CHECK_ARG(fp8 || in_dtype == FA4CP_DTYPE_BF16 || in_dtype == FA4CP_DTYPE_F16,
                  "input dtype must be f16, bf16 or e4m3");
  FA4CP_CHECK_ARG(fp8 || (q_descale == nullptr && k_descale == nullptr && v_descale == nullptr),
                  "descales apply to e4m3 inputs only");
  if (total_q == 0) return FA4CP_OK;
  FA4CP_CHECK_ARG(q && out && lse && k_pages && v_pages, "null tensor pointer");
  FA4CP_CHECK_ARG(aligned16(q) && aligned16(k_pages) && aligned16(v_pages) && aligned16(out),
                  "q, the page pools and out must be 16-byte aligned");
  Params p{};
  p.cu_q = cu_q;
  p.cu_k = cu_k;
  p.out = out;
  p.lse = lse;
  p.q_descale = q_descale;
  p.k_descale = k_descale;
  p.v_descale = v_descale;
  p.nseq = nseq;
  p.Hq = num_heads_q;
  p.Hkv = num_heads_kv;
  p.group = num_heads_q / num_heads_kv;
  p.pattern = FA4CP_PATTERN_VARLEN;
  p.causal = causal ? 1 : 0;
  p.accumulate = 0;
  p.in_fmt = in_dtype == FA4CP_DTYPE_BF16 ? 1 : 0;
  p.out_bf16 = out_dtype == FA4CP_DTYPE_BF16 ? 1 : 0;
  p.scale_log2 = softmax_scale * kLog2e;
  p.debug_withhold_kv = -1;
  p.block_table = block_table;
  p.page_size = page_size;
  p.max_pages = max_pages_per_seq;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (fp8) {
    FA4CP_CHECK_ARG(out_dtype == FA4CP_DTYPE_BF16, "e4m3 inputs produce a bf16 output");
    if (head_dim == 128)
      return launch2_paged<Traits2<128, 128, 3, true>>(q, k_pages, v_pages, num_pages, total_q,
                                                        max_seqlen_q, p, st);
  } else {
    if (head_dim == 128)
      return launch2_paged<Traits2<128, 128, 2, false>>(q, k_pages, v_pages, num_pages, total_q,
                                                         max_seqlen_q, p, st);
    if (head_dim == 64)
      return launch2_paged<Traits2<64, 128, 3, false>>(q, k_pages, v_pages, num_pages, total_q,
                                                        max_seqlen_q, p, st);
  }
  set_last_error("paged K/V takes head_dim 64 or 128 (f16 / bf16) or 128 (e4m3); got %d",
                 head_dim);
  return FA4CP_ERR_UNSUPPORTED;
}

extern "C" int fa4cp_device_status(int32_t* status, int32_t clear) {
  FA4CP_CHECK_ARG(status != nullptr, "status must not be NULL");
  FA4CP_CHECK_CUDA(cudaDeviceSynchronize());
  int v = 0;
  FA4CP_CHECK_CUDA(cudaMemcpyFromSymbol(&v, g_attn_status, sizeof(int)));
  if (clear) {
    int z = 0;
    FA4CP_CHECK_CUDA(cudaMemcpyToSymbol(g_attn_status, &z, sizeof(int)));
  }
  *status = v;
  return FA4CP_OK;
}

extern "C" int64_t fa4cp_attn_kv8_workspace_bytes(int64_t total_k, int32_t num_heads_kv,
                                                  int32_t head_dim) {
  if (total_k < 0 || num_heads_kv <= 0 || head_dim <= 0) return -1;
  const int64_t per_row = int64_t(4) * num_heads_kv * head_dim;  // bf16 K and V of one row
  if (total_k > INT64_MAX / per_row) return -1;                   // the size would overflow
  return total_k * per_row;
}

extern "C" int fa4cp_attn_fwd_kv8(const void* q, const void* k8, const void* v8, void* out,
                                  float* lse, const int32_t* cu_q, const int32_t* cu_k,
                                  int32_t nseq, int32_t max_seqlen_q, int64_t total_q,
                                  int64_t total_k, int32_t num_heads_q, int32_t num_heads_kv,
                                  int32_t head_dim, int32_t q_dtype, int32_t pattern,
                                  int32_t causal, float softmax_scale, const float* k_descale,
                                  const float* v_descale, int32_t accumulate, void* workspace,
                                  int64_t workspace_bytes, void* stream) {
  FA4CP_CHECK_ARG(q_dtype == FA4CP_DTYPE_BF16 || q_dtype == FA4CP_DTYPE_F16,
                  "kv8 attention takes an f16 or bf16 query");
  FA4CP_CHECK_ARG(num_heads_kv > 0 && head_dim > 0 && total_k >= 0, "bad sizes");
  const int64_t need = fa4cp_attn_kv8_workspace_bytes(total_k, num_heads_kv, head_dim);
  FA4CP_CHECK_ARG(need >= 0, "K/V of %lld x %d x %d elements: the workspace size overflows",
                  (long long)total_k, num_heads_kv, head_dim);
  FA4CP_CHECK_ARG(workspace_bytes >= need, "workspace too small: %lld < %lld bytes",
                  (long long)workspace_bytes, (long long)need);
  FA4CP_CHECK_ARG(need == 0 || workspace != nullptr, "workspace is NULL");
  FA4CP_CHECK_ARG(q_dtype == FA4CP_DTYPE_BF16, "kv8 attention converts K/V to bf16; use a bf16 query");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* kb = static_cast<uint8_t*>(workspace);
  uint8_t* vb = kb + need / 2;
  if (total_k > 0) {
    // e4m3 -> bf16 is exact (3 mantissa bits, exponents inside bf16's range); the descales
    // stay fp32 and the kernel applies them to the scores and to O
    int rc = launch_dequant_e4m3(k8, nullptr, kb, total_k, num_heads_kv, head_dim, st);
    if (rc) return rc;
    rc = launch_dequant_e4m3(v8, nullptr, vb, total_k, num_heads_kv, head_dim, st);
    if (rc) return rc;
  }
  return attn_fwd_impl(q, kb, vb, out, lse, cu_q, cu_k, nseq, max_seqlen_q, total_q, total_k,
                       num_heads_q, num_heads_kv, head_dim, q_dtype, q_dtype, pattern, causal,
                       softmax_scale, nullptr, k_descale, v_descale, accumulate, stream);
}

extern "C" int fa4cp_selftest_wait_expiry(const void* q, const void* k, const void* v, void* out,
                                          float* lse, const int32_t* cu, int32_t seqlen,
                                          int32_t* status_out, void* stream) {
  FA4CP_CHECK_ARG(seqlen >= 1 && seqlen <= 4096, "seqlen must be in [1, 4096]");
  FA4CP_CHECK_ARG(q && k && v && out && lse && cu && status_out, "null pointer");
  FA4CP_CHECK_ARG(aligned16(q) && aligned16(k) && aligned16(v) && aligned16(out),
                  "tensors must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int zero = 0;
  FA4CP_CHECK_CUDA(cudaStreamSynchronize(st));
  FA4CP_CHECK_CUDA(cudaMemcpyToSymbol(g_attn_status, &zero, sizeof(int)));
  Params p{};
  p.cu_q = cu;
  p.cu_k = cu;
  p.out = out;
  p.lse = lse;
  p.nseq = 1;
  p.Hq = 1;
  p.Hkv = 1;
  p.group = 1;
  p.pattern = FA4CP_PATTERN_VARLEN;
  p.causal = 1;
  p.in_fmt = 1;
  p.out_bf16 = 1;
  p.scale_log2 = kLog2e / sqrtf(128.0f);
  p.debug_withhold_kv = 0;  // the consumer's wait for K tile 0 can only run out
  int rc = launch2<Traits2<128, 128, 2, false>>(q, k, v, seqlen, seqlen, seqlen, p, st);
  if (rc) return rc;
  FA4CP_CHECK_CUDA(cudaStreamSynchronize(st));
  int observed = 0;
  FA4CP_CHECK_CUDA(cudaMemcpyFromSymbol(&observed, g_attn_status, sizeof(int)));
  FA4CP_CHECK_CUDA(cudaMemcpyToSymbol(g_attn_status, &zero, sizeof(int)));
  *status_out = observed;
  return FA4CP_OK;
}
