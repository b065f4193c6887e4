// Persistent ring kernel: a rank's whole zig-zag ring forward in one launch.
//
// Included into attn_fwd_sm100.cu (inside its anonymous namespace): it shares the two-tile
// traits, the barrier helpers, the error codes and the device status word of the per-step
// kernel, whose warp roles, TMEM plan (S0 | S1 | O0 | O1) and softmax it follows.  What
// changes is the K/V a CTA walks.  A CTA owns two 128-row query tiles of one half (early
// or late) of one local sequence and one query head; its K/V sequence is the concatenation
// of every ring step's K/V for those rows, in step order (reference
// fa4_ring/ring_attention.py:109-166):
//   step 0      the local K/V, causal (early half: keys [0, h); late half: keys [0, 2h));
//   1 <= s <= rank   the front half [0, h) of the K/V of rank (rank - s) mod S (slot s-1);
//   s > rank         all of it, [0, 2h), for late-half rows only.
// The online softmax runs across the whole sequence, so out and lse are written once: no
// per-step partial, merge or launch.  e4m3: the K and V descales belong to the source rank,
// so they change at step boundaries.  The running max is kept in scaled (log2) units, and O is
// kept in units of the current step's V descale: entering a step whose V descale differs,
// the softmax warps rescale O by old / new (together with any lazy max rescale), and the
// epilogue multiplies by the last one.  Both query tiles of a CTA walk the same number of K/V
// tiles: at the end of step 0 the lower tile walks one tile past its diagonal, which the
// causal mask zeroes.  Before the producer's first load of slot s-1 it waits (bounded) until
// that slot's arrival flag says it is present (RingFusedParams::arrived).
#pragma once

struct RingFusedParams {
  const int32_t* cu;          // local cu [nseq + 1] (every length even)
  void* out;                  // [total, Hq, D], q dtype
  float* lse;                 // [total, Hq]
  // arrival of the receive slots, or nullptr (all slots present): slot s-1 is present once
  // arrived[(s-1) * arrived_stride] >= arrived_base + s * arrived_step -- one hop counter for
  // the chained rotation (stride 0, step 1), or one flag per slot holding the call number for
  // the direct pushes (stride 1, step 0)
  const uint32_t* arrived;
  uint32_t arrived_base;
  int arrived_stride, arrived_step;
  // one-tile kernel only: first_step 1 walks the remote steps alone (step 0 ran in a launch of
  // its own, which wrote out / lse); accumulate 1 merges the result into out / lse
  int first_step, accumulate;
  int nseq, Hq, Hkv, group, S, rank;
  int n_pairs;                // query-tile pairs per half, max over sequences
  int n_tiles;                // tiles of the schedule (ring_grid); the grid walks them
  int in_fmt, out_bf16;
  float scale_log2;
  // e4m3 only: q descale [Hkv]; k / v descales [S, Hkv] indexed by SOURCE rank (nullptr: 1)
  const float* q_descale;
  const float* k_descales;
  const float* v_descales;
  unsigned long long arrive_wait_ns;  // bound of the wait for a hop counter
};

constexpr int kErrArrived = kErrDrain + 1;

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait of one thread for a hop counter written by a peer GPU (a stream write through
// NVLink): acquire at system scope, then order the CTA's later async-proxy (TMA) reads of
// the slot after it.  The bound is wall time (default 10 s, fa4cp_ring_set_wait_timeout_ms):
// it allows for host skew between ranks, and a dead peer still ends the wait.
__device__ __forceinline__ bool wait_arrived(const uint32_t* ctr, uint32_t target,
                                             unsigned long long limit_ns, volatile int* abort,
                                             int* status) {
  const unsigned long long t0 = global_ns();
  for (uint32_t it = 0;; ++it) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(ctr) : "memory");
    if (int32_t(v - target) >= 0) {
      asm volatile("fence.proxy.async.global;" ::: "memory");
      return true;
    }
    if (*abort) return false;
    if ((it & 15u) == 0 && *reinterpret_cast<volatile int*>(status) != 0) {
      *abort = 1;
      return false;
    }
    if (global_ns() - t0 > limit_ns) {
      *abort = 1;
      atomicCAS(status, 0, kErrArrived);
      return false;
    }
    __nanosleep(256);
  }
}

struct RingTile {
  int seq, half, pair, head, kvh;
};

// CTA order: all late-half pairs (they carry every step s > rank, the heavy tiles) before
// any early-half pair; within a half, pairs latest first (heaviest step 0), in chunks of
// kQtileChunk, inside a chunk by sequence, kv head, pair, query head of the GQA group (the
// kv-head grouping keeps the K/V of the CTAs in flight in L2).  Measured on one GPU with
// cfg2 shapes at cp=8: the slowest rank's launch 1.104 -> 1.058 ms against chunks that mix
// the two halves.
__device__ __forceinline__ bool ring_tile(const RingFusedParams& p, int tile, RingTile& w) {
  const int ch = min(kQtileChunk, p.n_pairs);
  const int chunks_per_half = (p.n_pairs + ch - 1) / ch;
  const int per_seq = ch * p.Hq;
  const int per_chunk = per_seq * p.nseq;
  int chunk = tile / per_chunk;
  int r = tile - chunk * per_chunk;
  const int round = chunk / chunks_per_half;  // 0: late half, 1: early half
  chunk -= round * chunks_per_half;
  const int seq = r / per_seq;
  r -= seq * per_seq;
  const int kvh = r / (ch * p.group);
  const int r2 = r - kvh * (ch * p.group);
  const int qd = chunk * ch + r2 / p.group;
  if (qd >= p.n_pairs || round > 1) return false;
  w.seq = seq;
  w.half = 1 - round;
  w.pair = p.n_pairs - 1 - qd;
  w.head = kvh * p.group + r2 % p.group;
  w.kvh = kvh;
  return true;
}

inline unsigned ring_grid(int n_pairs, int Hq, int nseq) {
  const int ch = n_pairs < kQtileChunk ? n_pairs : kQtileChunk;
  return unsigned(2 * ((n_pairs + ch - 1) / ch) * ch * Hq * nseq);
}

// K/V geometry of one CTA: step 0 (local, causal) then steps 1 .. S-1
struct RingSegs {
  int a, hh, half;      // sequence start, half length, 0 early / 1 late
  int k0_len, diag;     // step 0: keys [0, k0_len), key j visible to row i iff j <= i + diag
  int n0;               // K/V tiles of step 0 (up to the pair's last row)
  int S, rank;
  __device__ int len(int s) const {
    if (s == 0) return k0_len;
    return s <= rank ? hh : (half ? 2 * hh : 0);
  }
  __device__ int tiles(int s, int BN) const { return s == 0 ? n0 : (len(s) + BN - 1) / BN; }
};

// Walks the flat K/V tile index j through the steps (j only grows).
struct SegCursor {
  int s = 0, first = 0, count = 0;
  __device__ void start(const RingSegs& g, int BN) { s = 0; first = 0; count = g.tiles(0, BN); }
  __device__ void seek(const RingSegs& g, int j, int BN) {
    while (j >= first + count) {
      first += count;
      ++s;
      count = g.tiles(s, BN);
    }
  }
};

// Everything a CTA needs about one tile: its place, its steps' K/V and its two query tiles.
struct RingTileGeo {
  RingTile w;
  RingSegs g;
  int q_start, q0, rows_t[2], n_t[2];
};

__device__ __forceinline__ bool ring_tile_geo(const RingFusedParams& p, int tile, int BN,
                                              RingTileGeo& x) {
  if (!ring_tile(p, tile, x.w)) return false;  // padding of the schedule
  x.g.a = p.cu[x.w.seq];
  const int L = p.cu[x.w.seq + 1] - x.g.a;
  x.g.hh = L / 2;
  x.g.half = x.w.half;
  x.g.S = p.S;
  x.g.rank = p.rank;
  x.q_start = x.g.a + x.w.half * x.g.hh;
  const int q_len = x.w.half ? L - x.g.hh : x.g.hh;
  x.q0 = x.w.pair * 2 * BM;
  if (x.q0 >= q_len) return false;  // past this sequence's half
#pragma unroll
  for (int t = 0; t < 2; ++t) x.rows_t[t] = max(0, min(BM, q_len - (x.q0 + t * BM)));
  x.g.k0_len = x.w.half ? L : x.g.hh;
  x.g.diag = x.g.k0_len - q_len;
  const int kv_end0 = min(x.g.k0_len, x.q0 + x.rows_t[0] + x.rows_t[1] + x.g.diag);
  x.g.n0 = (kv_end0 + BN - 1) / BN;
  int n = 0;
  for (int s = 0; s < p.S; ++s) n += x.g.tiles(s, BN);
#pragma unroll
  for (int t = 0; t < 2; ++t) x.n_t[t] = x.rows_t[t] > 0 ? n : 0;
  return true;
}

// e4m3 only: every K/V tile of a CTA goes to the PV MMA as two e4m3 terms (fp8_p_to_tmem)
// when a row of its query tiles sees fewer than 128 keys over the whole ring -- the first row
// of the lower query tile: step 0 (causal) plus every remote step.  Over few keys the rounding
// of an e4m3 P does not average out; only the first early-half pair of rank 0 and the pairs of
// tiny sequences qualify; they run in the kernel's split pass (SPLIT_PASS), the rest in the
// main pass.  All three roles of both passes evaluate it alike.
__device__ __forceinline__ bool ring_split_all(const RingTileGeo& x, int S) {
  // sum of RingSegs::len(s) over s = 1 .. S-1: h for s <= rank, 2h (late half) or 0 after
  const int64_t remote = int64_t(x.g.rank) * x.g.hh +
                         (x.g.half ? int64_t(S - 1 - x.g.rank) * 2 * x.g.hh : 0);
  return int64_t(x.q0) + x.g.diag + 1 + remote < 128;
}

// One tile per CTA (f16 / bf16): the straight-line form, measured 3% faster than the tile
// loop below run for a single tile.
template <class TR>
__global__ void __launch_bounds__(TR::THREADS, 1)
    ring_fused_kernel(const __grid_constant__ CUtensorMap tmQ,
                      const __grid_constant__ CUtensorMap tmK0,
                      const __grid_constant__ CUtensorMap tmV0,
                      const __grid_constant__ CUtensorMap tmKs,
                      const __grid_constant__ CUtensorMap tmVs, const RingFusedParams p) {
  static_assert(!TR::PERSISTENT && !TR::FP8, "the one-tile ring kernel (f16 / bf16)");
  constexpr int D = TR::D, BN = TR::BN, ST = TR::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  RingTileGeo x;
  if (!ring_tile_geo(p, int(blockIdx.x), BN, x)) return;  // uniform, before any set-up
  const RingTile w = x.w;
  const RingSegs g = x.g;
  const int q_start = x.q_start, q0 = x.q0;
  const int rows_t[2] = {x.rows_t[0], x.rows_t[1]};
  // remote-only walk (first_step 1): the tiles of step 0 are skipped; j counts the walked tiles
  // (pipeline stages and phases), j + j0 is the tile in the CTA's K/V sequence
  const int j0 = p.first_step ? g.n0 : 0;
  const int n_t[2] = {x.n_t[0] > j0 ? x.n_t[0] - j0 : 0, x.n_t[1] > j0 ? x.n_t[1] - j0 : 0};

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
  auto p_full = [&](int t) { return BAR(9 + 4 * ST + t * TR::P_SPLIT); };
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
    for (int t = 0; t < 2; ++t) {
      mbar_init(s_full(t), 1);
      mbar_init(p_full(t), 128);
      mbar_init(o_done(t), 1);
    }
    mbar_init(td_bar, 1);
    *abort = 0;
    fence_mbar_init();
  }
  if (warp == 8 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK0);
    tma_prefetch_desc(&tmV0);
    tma_prefetch_desc(&tmKs);
    tma_prefetch_desc(&tmVs);
  }
  if (warp == 9) {
    tmem_alloc(smem_u32(tmem_slot), TR::TM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp >= 8) {
   setmaxnreg_dec<TR::REGS_PRODUCER>();
   if (warp == 8) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const uint64_t pol_kv = policy_evict_last();
      int last_k[ST], last_v[ST];
      for (int s = 0; s < ST; ++s) last_k[s] = last_v[s] = -1;
      const int nmax = max(n_t[0], n_t[1]);
      mbar_arrive_expect_tx(q_full, 2 * TR::Q_TILE_BYTES);
#pragma unroll
      for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int c = 0; c < TR::NCH; ++c)
          tma_load_3d(smem_u32(smem + TR::OFF_Q + t * TR::Q_TILE_BYTES + c * TR::Q_CHUNK_BYTES),
                      &tmQ, c * TR::CHUNK, w.head, q_start + q0 + t * BM, q_full);
      SegCursor cur;
      cur.start(g, BN);
      int waited = 0;  // highest step whose slot is known present
      for (int j = 0; j < nmax; ++j) {
        cur.seek(g, j + j0, BN);
        const int s = j % ST, ph = (j / ST) & 1;
        const int row = g.a + (j + j0 - cur.first) * BN;
        if (cur.s > waited) {
          if (p.arrived != nullptr &&
              !wait_arrived(p.arrived + (cur.s - 1) * p.arrived_stride,
                            p.arrived_base + uint32_t(cur.s * p.arrived_step), p.arrive_wait_ns,
                            abort, status))
            break;
          waited = cur.s;
        }
        if (j >= ST && !mbar_wait(k_empty(s), ph ^ 1, abort, kErrKEmpty, status)) break;
        mbar_arrive_expect_tx(k_full(s), TR::KV_BYTES);
#pragma unroll
        for (int c = 0; c < TR::NCH; ++c) {
          const uint32_t dst = smem_u32(smem + TR::OFF_K + s * TR::KV_BYTES + c * TR::KV_CHUNK_BYTES);
          if (cur.s == 0)
            tma_load_3d_hint(dst, &tmK0, c * TR::CHUNK, w.kvh, row, k_full(s), pol_kv);
          else
            tma_load_4d_hint(dst, &tmKs, c * TR::CHUNK, w.kvh, row, cur.s - 1, k_full(s), pol_kv);
        }
        last_k[s] = j;
        if (j >= ST && !mbar_wait(v_empty(s), ph ^ 1, abort, kErrVEmpty, status)) break;
        mbar_arrive_expect_tx(v_full(s), TR::KV_BYTES);
#pragma unroll
        for (int c = 0; c < TR::NCH; ++c) {
          const uint32_t dst = smem_u32(smem + TR::OFF_V + s * TR::KV_BYTES + c * TR::KV_CHUNK_BYTES);
          if (cur.s == 0)
            tma_load_3d_hint(dst, &tmV0, c * TR::CHUNK, w.kvh, row, v_full(s), pol_kv);
          else
            tma_load_4d_hint(dst, &tmVs, c * TR::CHUNK, w.kvh, row, cur.s - 1, v_full(s), pol_kv);
        }
        last_v[s] = j;
      }
      // every copy this thread issued has landed before it leaves its role
      mbar_wait_drain(q_full, 0, kErrDrain, status);
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
      auto issue_pv = [&](int t, int stage, bool first) {
        const uint32_t sV = smem_u32(smem + TR::OFF_V + stage * TR::KV_BYTES);
#pragma unroll
        for (int kk = 0; kk < BN / TR::MMA_K; ++kk) {
          const uint64_t bdesc = make_desc_sw128(sV + kk * TR::MMA_K * 128, TR::KV_CHUNK_BYTES, 1024);
          const uint32_t a_tmem = tmem + uint32_t(TR::tm_s(t) + kk * 8);
          const uint32_t acc = (!first || kk > 0) ? 1u : 0u;
          if constexpr (TR::FP8)
            mma_f8_ts(tmem + uint32_t(TR::tm_o(t)), a_tmem, bdesc, idesc_pv, acc);
          else
            mma_f16_ts(tmem + uint32_t(TR::tm_o(t)), a_tmem, bdesc, idesc_pv, acc);
        }
      };
      const int nmax = max(n_t[0], n_t[1]);
      bool ok = mbar_wait(q_full, 0, abort, kErrQ, status);
      if (ok) tc_fence_after();
      if (ok && nmax > 0) {
        ok = mbar_wait(k_full(0), 0, abort, kErrKFull, status);
        if (ok) {
          tc_fence_after();
          if (n_t[0] > 0) issue_s(0, 0);
          if (n_t[1] > 0) issue_s(1, 0);
          tc_commit(k_empty(0));
        }
      }
      for (int j = 0; ok && j < nmax; ++j) {
        const int s = j % ST;
        bool v_ready = false, k_next_ready = false;
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          if (j >= n_t[t]) continue;
          if (!v_ready) {
            if (!mbar_wait(v_full(s), (j / ST) & 1, abort, kErrVFull, status)) { ok = false; break; }
            v_ready = true;
          }
          if (!mbar_wait(p_full(t), j & 1, abort, kErrPFull, status)) { ok = false; break; }
          tc_fence_after();
          issue_pv(t, s, j == 0);
          tc_commit(o_done(t));
          if (j + 1 < n_t[t]) {
            const int s1 = (j + 1) % ST;
            if (!k_next_ready) {
              if (!mbar_wait(k_full(s1), ((j + 1) / ST) & 1, abort, kErrKFull, status)) {
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
        if (k_next_ready) tc_commit(k_empty((j + 1) % ST));
      }
      // every MMA issued above has completed before TMEM is released
      tc_commit(td_bar);
      mbar_wait_drain(td_bar, 0, kErrDrain, status);
    }
   }
  } else {
    setmaxnreg_inc<TR::REGS_SOFTMAX>();
    // ------------------------------------------------------------ softmax + epilogue
    const int t = warp >> 2;  // query tile of this warpgroup
    const int wq = warp & 3;
    const int r = wq * 32 + lane;
    const uint32_t t_lane = tmem + (uint32_t(wq * 32) << 16);
    const int nn = n_t[t];
    if (nn > 0) {
      const int first = q0 + t * BM;
      const int key_lim = first + r + g.diag;  // step 0 only
      const float qd = (TR::FP8 && p.q_descale != nullptr) ? p.q_descale[w.kvh] : 1.0f;
      // score scale (log2 units) and V descale of step s: the descales of its source rank
      auto step_scales = [&](int s, float& sc, float& vs) {
        const int src = (p.rank - s + p.S) % p.S;
        sc = p.scale_log2 * qd;
        vs = 1.0f;
        if constexpr (TR::FP8) {
          if (p.k_descales != nullptr) sc *= p.k_descales[src * p.Hkv + w.kvh];
          if (p.v_descales != nullptr) vs = p.v_descales[src * p.Hkv + w.kvh];
        }
      };
      float scale, vscale;
      step_scales(0, scale, vscale);
      int step = 0;
      float m = kNegInf, l = 0.f;  // m: running max of the scaled scores (log2 units)
      bool aborted = false;
      SegCursor cur;
      cur.start(g, BN);

      for (int j = 0; j < nn; ++j) {
        cur.seek(g, j + j0, BN);
        float fo = 1.0f;  // O factor when the V descale changes with the step
        if (cur.s != step) {
          step = cur.s;
          float vs_new;
          step_scales(step, scale, vs_new);
          fo = vscale / vs_new;
          vscale = vs_new;
        }
        bool ok = mbar_wait(s_full(t), j & 1, abort, kErrSFull, status);
        if (!__all_sync(0xffffffffu, ok)) { aborted = true; break; }
        tc_fence_after();
        uint32_t sr[BN / 32][32];
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) tmem_ld32(t_lane + uint32_t(TR::tm_s(t) + c * 32), sr[c]);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) reg_fence32(sr[c]);

        const int kbase = (j + j0 - cur.first) * BN;
        const int seg_len = g.len(cur.s);
        const bool causal = cur.s == 0;
        const bool need_mask = (kbase + BN > seg_len) || (causal && kbase + BN - 1 > first + g.diag);
        if (need_mask) {
#pragma unroll
          for (int c = 0; c < BN / 32; ++c)
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              const int key = kbase + c * 32 + e;
              if (key >= seg_len || (causal && key > key_lim)) sr[c][e] = __float_as_uint(kNegInf);
            }
        }
        float mx4[4] = {kNegInf, kNegInf, kNegInf, kNegInf};
#pragma unroll
        for (int c = 0; c < BN / 32; ++c)
#pragma unroll
          for (int e = 0; e < 32; e += 2)
            mx4[c] = fmax3(mx4[c], __uint_as_float(sr[c][e]), __uint_as_float(sr[c][e + 1]));
        const float mx = fmax3(fmaxf(mx4[0], mx4[1]), mx4[2], mx4[3]) * scale;  // scale > 0
        const float m_new = fmaxf(m, mx);
        if (j == 0) {
          m = m_new;
        } else {
          const bool need = (m_new - m) > kRescaleThreshold;
          if (__any_sync(0xffffffffu, need) || fo != 1.0f) {  // fo is uniform in the CTA
            // PV_t(j-1) is complete: S_t(j) was issued after it and has completed.
            const float f = need ? ex2_approx(m - m_new) : 1.0f;
            if (need) { l *= f; m = m_new; }
            const uint64_t f2 = f2pack(f * fo, f * fo);
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
        const float neg_m = (m == kNegInf) ? 0.f : -m;
        const uint64_t negm2 = f2pack(neg_m, neg_m);
        const uint64_t scale2 = f2pack(scale, scale);
        uint64_t rs2[2] = {0ull, 0ull};
        // P in 64-key halves: exps of a half are kept (as fp32 bits, in place of S) for the
        // row sum, which is added up after P has been handed to the MMA warp
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
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(p_full(t));
#pragma unroll
        for (int c = 0; c < BN / 32; ++c)
#pragma unroll
          for (int e = 0; e < 32; e += 4) {
            rs2[0] = fadd2(rs2[0], f2pack(__uint_as_float(sr[c][e]), __uint_as_float(sr[c][e + 1])));
            rs2[1] = fadd2(rs2[1], f2pack(__uint_as_float(sr[c][e + 2]), __uint_as_float(sr[c][e + 3])));
          }
        const uint64_t rs = fadd2(rs2[0], rs2[1]);
        l += f2lo(rs) + f2hi(rs);
      }

      // ---------------------------------------------------------- epilogue
      if (!aborted) {
        bool ok = mbar_wait(o_done(t), (nn - 1) & 1, abort, kErrODone, status);
        aborted = !__all_sync(0xffffffffu, ok);
      }
      if (!aborted) {
        tc_fence_after();
        const bool valid = r < rows_t[t];
        const int64_t grow = int64_t(q_start) + first + r;
        const bool any_key = (m != kNegInf) && (l > 0.f);
        const float lse_new = any_key ? (m + lg2_approx(l)) * kLn2 : kNegInf;
        float* lse_ptr = p.lse + grow * p.Hq + w.head;
        // out = acc * ca + O_raw * cb (O is in units of the last V descale)
        float ca = 0.f, cb = any_key ? vscale / l : 0.f, lse_out = lse_new;
        bool write = valid, read_acc = false;
        if (valid && p.accumulate) {  // merge into the partial already in (out, lse)
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
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          tmem_ld32(t_lane + uint32_t(TR::tm_o(t) + c * 32), o);
          tmem_wait_ld();
          reg_fence32(o);
          if (write) {
            uint4* dst = reinterpret_cast<uint4*>(orow + c * 64);
            float f[32];
#pragma unroll
            for (int e = 0; e < 32; ++e) f[e] = __uint_as_float(o[e]) * cb;
            if (read_acc) {
#pragma unroll
              for (int v4 = 0; v4 < 4; ++v4) {
                const uint4 a = dst[v4];
                const uint32_t wa4[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                  float lo, hi;
                  if (p.out_bf16) {
                    lo = __uint_as_float(wa4[i] << 16);
                    hi = __uint_as_float(wa4[i] & 0xFFFF0000u);
                  } else {
                    const float2 tt = __half22float2(*reinterpret_cast<const __half2*>(&wa4[i]));
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
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 9) tmem_dealloc(tmem, TR::TM_COLS);
}

// ---------------------------------------------------------------------------
// One query tile per CTA (head_dim 256): S (64 keys) x 2 + O (256) fill 384 TMEM columns, so a
// CTA holds a single 128-row query tile, with the per-step single-tile kernel's roles (warps
// 0-3 softmax + epilogue, warp 4 TMA, warp 5 MMA) and the ring walk above.  ring_tile's
// "pair" is a 128-row query tile here (RingFusedParams::n_pairs counts query tiles per half).
// f16 / bf16 operands; descales (per source rank, as the e4m3 kernel) are for K/V that are
// the exact f16 / bf16 images of e4m3 values: the score scale of a step is
// scale * q_descale * k_descale[src], and O is kept in units of the current step's V descale
// (rescaled by old / new on entering a step, the epilogue multiplies by the last one).
// Reference: the bf16-Q x e4m3-K/V ring of fa4_ring/ring_attention.py:139-166 with the
// descales of fa4_ring/fa4_backend.py:99-120.
struct RingTileGeo1 {
  RingTile w;
  RingSegs g;
  int q_start, q0, rows, n;
};

__device__ __forceinline__ bool ring_tile_geo1(const RingFusedParams& p, int tile, int BN,
                                               RingTileGeo1& x) {
  if (!ring_tile(p, tile, x.w)) return false;  // padding of the schedule
  x.g.a = p.cu[x.w.seq];
  const int L = p.cu[x.w.seq + 1] - x.g.a;
  x.g.hh = L / 2;
  x.g.half = x.w.half;
  x.g.S = p.S;
  x.g.rank = p.rank;
  x.q_start = x.g.a + x.w.half * x.g.hh;
  const int q_len = x.w.half ? L - x.g.hh : x.g.hh;
  x.q0 = x.w.pair * BM;
  if (x.q0 >= q_len) return false;  // past this sequence's half
  x.rows = min(BM, q_len - x.q0);
  x.g.k0_len = x.w.half ? L : x.g.hh;
  x.g.diag = x.g.k0_len - q_len;
  const int kv_end0 = min(x.g.k0_len, x.q0 + x.rows + x.g.diag);  // >= 1
  x.g.n0 = (kv_end0 + BN - 1) / BN;
  int n = 0;
  for (int s = 0; s < p.S; ++s) n += x.g.tiles(s, BN);
  x.n = n;
  return true;
}

template <class TR>
__global__ void __launch_bounds__(kThreads, 1)
    ring_fused_1q_kernel(const __grid_constant__ CUtensorMap tmQ,
                         const __grid_constant__ CUtensorMap tmK0,
                         const __grid_constant__ CUtensorMap tmV0,
                         const __grid_constant__ CUtensorMap tmKs,
                         const __grid_constant__ CUtensorMap tmVs, const RingFusedParams p) {
  static_assert(!TR::FP8, "the one-query-tile ring kernel takes f16 / bf16 operands");
  constexpr int D = TR::D, BN = TR::BN, ST = TR::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  RingTileGeo1 x;
  if (!ring_tile_geo1(p, int(blockIdx.x), BN, x)) return;  // uniform, before any set-up
  const RingTile w = x.w;
  const RingSegs g = x.g;
  const int q0 = x.q0, rows = x.rows, n_kv = x.n;

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
  // PV_i commits o_done(i & 1), as in the per-step single-tile kernel
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
    tma_prefetch_desc(&tmK0);
    tma_prefetch_desc(&tmV0);
    tma_prefetch_desc(&tmKs);
    tma_prefetch_desc(&tmVs);
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
        tma_load_3d(smem_u32(smem + TR::OFF_Q + c * TR::Q_CHUNK_BYTES), &tmQ, c * TR::CHUNK,
                    w.head, x.q_start + q0, q_full);
      // the step of tile j and its first K/V row, advanced at step boundaries only
      int step = 0, step_end = g.tiles(0, BN), row = g.a - BN;
      for (int j = 0; j < n_kv; ++j) {
        row += BN;
        if (j == step_end) {  // next step with tiles (steps without any are skipped)
          do {
            ++step;
            step_end += g.tiles(step, BN);
          } while (j >= step_end);
          row = g.a;
          if (p.arrived != nullptr &&
              !wait_arrived(p.arrived + (step - 1) * p.arrived_stride,
                            p.arrived_base + uint32_t(step * p.arrived_step), p.arrive_wait_ns,
                            abort, status))
            break;
        }
        const int s = j % ST, ph = (j / ST) & 1;
        if (j >= ST && !mbar_wait(k_empty(s), ph ^ 1, abort, kErrKEmpty, status)) break;
        mbar_arrive_expect_tx(k_full(s), TR::KV_BYTES);
#pragma unroll
        for (int c = 0; c < TR::NCH; ++c) {
          const uint32_t dst = smem_u32(smem + TR::OFF_K + s * TR::KV_BYTES + c * TR::KV_CHUNK_BYTES);
          if (step == 0)
            tma_load_3d_hint(dst, &tmK0, c * TR::CHUNK, w.kvh, row, k_full(s), pol_kv);
          else
            tma_load_4d_hint(dst, &tmKs, c * TR::CHUNK, w.kvh, row, step - 1, k_full(s), pol_kv);
        }
        last_k[s] = j;
        if (j >= ST && !mbar_wait(v_empty(s), ph ^ 1, abort, kErrVEmpty, status)) break;
        mbar_arrive_expect_tx(v_full(s), TR::KV_BYTES);
#pragma unroll
        for (int c = 0; c < TR::NCH; ++c) {
          const uint32_t dst = smem_u32(smem + TR::OFF_V + s * TR::KV_BYTES + c * TR::KV_CHUNK_BYTES);
          if (step == 0)
            tma_load_3d_hint(dst, &tmV0, c * TR::CHUNK, w.kvh, row, v_full(s), pol_kv);
          else
            tma_load_4d_hint(dst, &tmVs, c * TR::CHUNK, w.kvh, row, step - 1, v_full(s), pol_kv);
        }
        last_v[s] = j;
      }
      // every copy this thread issued has landed before it leaves its role
      mbar_wait_drain(q_full, 0, kErrDrain, status);
      for (int s = 0; s < ST; ++s) {
        if (last_k[s] >= 0) mbar_wait_drain(k_full(s), (last_k[s] / ST) & 1, kErrDrain, status);
        if (last_v[s] >= 0) mbar_wait_drain(v_full(s), (last_v[s] / ST) & 1, kErrDrain, status);
      }
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const int fmt = p.in_fmt;
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
    const int key_lim = q0 + r + g.diag;  // step 0 only
    const float qd = p.q_descale != nullptr ? p.q_descale[w.kvh] : 1.0f;
    // score scale (log2 units) and V descale of step s: the descales of its source rank
    auto step_scales = [&](int s, float& sc, float& vs) {
      const int src = (p.rank - s + p.S) % p.S;
      sc = p.scale_log2 * qd;
      vs = 1.0f;
      if (p.k_descales != nullptr) sc *= p.k_descales[src * p.Hkv + w.kvh];
      if (p.v_descales != nullptr) vs = p.v_descales[src * p.Hkv + w.kvh];
    };
    float scale, vscale;
    step_scales(0, scale, vscale);
    // the step of tile j, its key length and tile j's first key within it, advanced at step
    // boundaries only (CTA-uniform)
    int step = 0, step_end = g.tiles(0, BN), seg_len = g.len(0), kbase = -BN;
    float m = kNegInf, l = 0.f;  // m: running max of the scaled scores (log2 units)
    bool aborted = false;

    for (int j = 0; j < n_kv; ++j) {
      kbase += BN;
      float fo = 1.0f;  // O factor when the V descale changes with the step
      if (j == step_end) {
        do {
          ++step;
          step_end += g.tiles(step, BN);
        } while (j >= step_end);
        seg_len = g.len(step);
        kbase = 0;
        float vs_new;
        step_scales(step, scale, vs_new);
        fo = vscale / vs_new;
        vscale = vs_new;
      }
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

      const bool causal = step == 0;
      const bool need_mask = (kbase + BN > seg_len) || (causal && kbase + BN - 1 > q0 + g.diag);
      if (need_mask) {
#pragma unroll
        for (int c = 0; c < BN / 32; ++c)
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const int key = kbase + c * 32 + e;
            if (key >= seg_len || (causal && key > key_lim)) sr[c][e] = __float_as_uint(kNegInf);
          }
      }
      float mx = kNegInf;
#pragma unroll
      for (int c = 0; c < BN / 32; ++c)
#pragma unroll
        for (int e = 0; e < 32; ++e) mx = fmaxf(mx, __uint_as_float(sr[c][e]));
      const float m_new = fmaxf(m, mx * scale);  // scale > 0
      if (j == 0) {
        m = m_new;
      } else {
        const bool need = (m_new - m) > kRescaleThreshold;
        if (__any_sync(0xffffffffu, need) || fo != 1.0f) {
          const float f = need ? ex2_approx(m - m_new) : 1.0f;
          if (need) { l *= f; m = m_new; }
          // PV_{j-1} has completed before O is rescaled
          ok = mbar_wait(o_done((j - 1) & 1), ((j - 1) >> 1) & 1, abort, kErrODone, status);
          if (!__all_sync(0xffffffffu, ok)) { aborted = true; break; }
          tc_fence_after();
          const float fof = f * fo;
#pragma unroll 1
          for (int c = 0; c < D / 32; ++c) {
            uint32_t o[32];
            tmem_ld32(t_lane + uint32_t(TR::TM_O + c * 32), o);
            tmem_wait_ld();
            reg_fence32(o);
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * fof);
            tmem_st32(t_lane + uint32_t(TR::TM_O + c * 32), o);
          }
          tmem_wait_st();
        }
      }
      const float neg_m = (m == kNegInf) ? 0.f : -m;
      float rs = 0.f;
#pragma unroll
      for (int half = 0; half < BN / 64; ++half) {
        uint32_t pw[32];
#pragma unroll
        for (int e = 0; e < 64; e += 2) {
          const int c = half * 2 + (e >> 5), ee = e & 31;
          const float x0 = ex2_approx(fmaf(__uint_as_float(sr[c][ee]), scale, neg_m));
          const float x1 = ex2_approx(fmaf(__uint_as_float(sr[c][ee + 1]), scale, neg_m));
          rs += x0 + x1;
          pw[e >> 1] = p.in_fmt ? pack_bf16x2(x0, x1) : pack_f16x2(x0, x1);
        }
        tmem_st32(t_lane + uint32_t(b * BN + half * 32), pw);
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
    if (!aborted) {  // warp-uniform: every lane takes part in the TMEM loads
      const bool valid = r < rows;
      const int64_t grow = int64_t(x.q_start) + q0 + r;
      const bool any_key = (m != kNegInf) && (l > 0.f);
      const float cb = any_key ? vscale / l : 0.f;
      uint8_t* orow = static_cast<uint8_t*>(p.out) + (grow * p.Hq + w.head) * int64_t(D) * 2;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        tmem_ld32(t_lane + uint32_t(TR::TM_O + c * 32), o);
        tmem_wait_ld();
        reg_fence32(o);
        if (valid) {
          uint4* dst = reinterpret_cast<uint4*>(orow + c * 64);
#pragma unroll
          for (int v4 = 0; v4 < 4; ++v4) {
            uint32_t wd[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float f0 = __uint_as_float(o[v4 * 8 + 2 * i]) * cb;
              const float f1 = __uint_as_float(o[v4 * 8 + 2 * i + 1]) * cb;
              wd[i] = p.out_bf16 ? pack_bf16x2(f0, f1) : pack_f16x2(f0, f1);
            }
            dst[v4] = make_uint4(wd[0], wd[1], wd[2], wd[3]);
          }
        }
      }
      if (valid) p.lse[grow * p.Hq + w.head] = any_key ? (m + lg2_approx(l)) * kLn2 : kNegInf;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 5) tmem_dealloc(tmem, TR::TM_COLS);
}

// Persistent form (e4m3): one CTA per SM walks the heaviest-first tile list (static
// boustrophedon schedule), with the per-step kernel's cross-tile hand-offs: the Q buffers are
// refilled once the previous tile's S MMAs completed (q_empty), and PV_t of a new tile waits
// until the previous tile's epilogue has read O_t (o_free).  Measured on one GPU (cfg3
// shapes): 6% faster than one tile per CTA.
// e4m3 runs in two passes over the same tile list: SPLIT_PASS = false takes every tile whose
// rows all see 128 or more keys and SPLIT_PASS = true the few others (ring_split_all), with
// every P split into two e4m3 terms.  The split code lives only in the second instantiation:
// compiled into the main kernel, even unused, it cost 5.6% (cfg3 ring shapes).
template <class TR, bool SPLIT_PASS>
__global__ void __launch_bounds__(TR::THREADS, 1)
    ring_fused_persistent_kernel(const __grid_constant__ CUtensorMap tmQ,
                      const __grid_constant__ CUtensorMap tmK0,
                      const __grid_constant__ CUtensorMap tmV0,
                      const __grid_constant__ CUtensorMap tmKs,
                      const __grid_constant__ CUtensorMap tmVs, const RingFusedParams p) {
  static_assert(TR::PERSISTENT, "the persistent ring kernel");
  constexpr int D = TR::D, BN = TR::BN, ST = TR::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tiles = p.n_tiles;
  // one tile per CTA, or (persistent) a static boustrophedon walk over the heaviest-first
  // tile list with a stride of the grid: round k forward when k is even, backward when odd
  const int G = int(gridDim.x);
  auto snake_tile = [&](int k) -> int {
    return k * G + ((k & 1) ? G - 1 - int(blockIdx.x) : int(blockIdx.x));
  };
  // the tiles of this pass (e4m3: split or not, ring_split_all; otherwise all)
  auto in_pass = [&](const RingTileGeo& x) -> bool {
    if constexpr (TR::FP8) return ring_split_all(x, p.S) == SPLIT_PASS;
    return true;
  };
  static_assert(TR::FP8 || !SPLIT_PASS, "only e4m3 has a split pass");

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
  auto p_full = [&](int t) { return BAR(9 + 4 * ST + t * TR::P_SPLIT); };
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
      mbar_init(p_full(t), 128);
      mbar_init(o_done(t), 1);
      mbar_init(o_free(t), 128);
    }
    mbar_init(td_bar, 1);
    *abort = 0;
    fence_mbar_init();
  }
  if (warp == 8 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK0);
    tma_prefetch_desc(&tmV0);
    tma_prefetch_desc(&tmKs);
    tma_prefetch_desc(&tmVs);
  }
  if (warp == 9) {
    tmem_alloc(smem_u32(tmem_slot), TR::TM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp >= 8) {
   setmaxnreg_dec<TR::REGS_PRODUCER>();
   if (warp == 8) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const uint64_t pol_kv = policy_evict_last();
      int last_k[ST], last_v[ST];
      for (int s = 0; s < ST; ++s) last_k[s] = last_v[s] = -1;
      int kv_it = 0, tile_it = 0;
      int waited = 0;  // highest step whose slot is known present (the counter only grows)
      bool ok = true;
      for (int it_tile = 0, tile = snake_tile(0); (TR::PERSISTENT || it_tile == 0) && ok && tile < n_tiles; tile = snake_tile(++it_tile)) {
        RingTileGeo x;
        if (!ring_tile_geo(p, tile, BN, x) || !in_pass(x)) continue;
        // the Q buffers are free once every S MMA of the previous tile has completed
        if (tile_it > 0 && !mbar_wait(q_empty, (tile_it - 1) & 1, abort, kErrQ, status)) break;
        mbar_arrive_expect_tx(q_full, 2 * TR::Q_TILE_BYTES);
#pragma unroll
        for (int t = 0; t < 2; ++t)
#pragma unroll
          for (int c = 0; c < TR::NCH; ++c)
            tma_load_3d(smem_u32(smem + TR::OFF_Q + t * TR::Q_TILE_BYTES + c * TR::Q_CHUNK_BYTES),
                        &tmQ, c * TR::CHUNK, x.w.head, x.q_start + x.q0 + t * BM, q_full);
        SegCursor cur;
        cur.start(x.g, BN);
        const int nmax = max(x.n_t[0], x.n_t[1]);
        for (int j = 0; j < nmax; ++j, ++kv_it) {
          cur.seek(x.g, j, BN);
          const int s = kv_it % ST, ph = (kv_it / ST) & 1;
          const int row = x.g.a + (j - cur.first) * BN;
          if (cur.s > waited) {
            if (p.arrived != nullptr &&
                !wait_arrived(p.arrived + (cur.s - 1) * p.arrived_stride,
                              p.arrived_base + uint32_t(cur.s * p.arrived_step), p.arrive_wait_ns,
                              abort, status)) { ok = false; break; }
            waited = cur.s;
          }
          if (kv_it >= ST && !mbar_wait(k_empty(s), ph ^ 1, abort, kErrKEmpty, status)) { ok = false; break; }
          mbar_arrive_expect_tx(k_full(s), TR::KV_BYTES);
#pragma unroll
          for (int c = 0; c < TR::NCH; ++c) {
            const uint32_t dst = smem_u32(smem + TR::OFF_K + s * TR::KV_BYTES + c * TR::KV_CHUNK_BYTES);
            if (cur.s == 0)
              tma_load_3d_hint(dst, &tmK0, c * TR::CHUNK, x.w.kvh, row, k_full(s), pol_kv);
            else
              tma_load_4d_hint(dst, &tmKs, c * TR::CHUNK, x.w.kvh, row, cur.s - 1, k_full(s), pol_kv);
          }
          last_k[s] = kv_it;
          if (kv_it >= ST && !mbar_wait(v_empty(s), ph ^ 1, abort, kErrVEmpty, status)) { ok = false; break; }
          mbar_arrive_expect_tx(v_full(s), TR::KV_BYTES);
#pragma unroll
          for (int c = 0; c < TR::NCH; ++c) {
            const uint32_t dst = smem_u32(smem + TR::OFF_V + s * TR::KV_BYTES + c * TR::KV_CHUNK_BYTES);
            if (cur.s == 0)
              tma_load_3d_hint(dst, &tmV0, c * TR::CHUNK, x.w.kvh, row, v_full(s), pol_kv);
            else
              tma_load_4d_hint(dst, &tmVs, c * TR::CHUNK, x.w.kvh, row, cur.s - 1, v_full(s), pol_kv);
          }
          last_v[s] = kv_it;
        }
        ++tile_it;
      }
      // every copy this thread issued has landed before it leaves its role
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
      auto issue_pv = [&](int t, int stage, bool first) {
        const uint32_t sV = smem_u32(smem + TR::OFF_V + stage * TR::KV_BYTES);
#pragma unroll
        for (int kk = 0; kk < BN / TR::MMA_K; ++kk) {
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
      int p_cnt[2] = {0, 0};       // P hand-offs consumed per query tile (p_full phases)
      int ofree_cnt[2] = {0, 0};   // epilogues that read O_t (o_free phases) ...
      int ofree_seen[2] = {0, 0};  // ... and how many of them this thread has waited for
      bool ok = true;
      for (int it_tile = 0, tile = snake_tile(0); (TR::PERSISTENT || it_tile == 0) && ok && tile < n_tiles; tile = snake_tile(++it_tile)) {
        RingTileGeo x;
        if (!ring_tile_geo(p, tile, BN, x) || !in_pass(x)) continue;
        const int nmax = max(x.n_t[0], x.n_t[1]);
        if (!mbar_wait(q_full, tile_it & 1, abort, kErrQ, status)) { ok = false; break; }
        tc_fence_after();
        if (nmax > 0) {
          const int s0 = kv_it % ST;
          if (!mbar_wait(k_full(s0), (kv_it / ST) & 1, abort, kErrKFull, status)) { ok = false; break; }
          tc_fence_after();
          if (x.n_t[0] > 0) issue_s(0, s0);
          if (x.n_t[1] > 0) issue_s(1, s0);
          tc_commit(k_empty(s0));
        }
        for (int j = 0; ok && j < nmax; ++j) {
          const int it = kv_it + j, s = it % ST;
          bool v_ready = false, k_next_ready = false;
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            if (j >= x.n_t[t]) continue;
            if (j == 0 && ofree_seen[t] < ofree_cnt[t]) {
              // PV_t(0) overwrites O_t: the previous tile's epilogue must have read it
              if (!mbar_wait(o_free(t), ofree_seen[t] & 1, abort, kErrODone, status)) { ok = false; break; }
              ++ofree_seen[t];
            }
            if (!v_ready) {
              if (!mbar_wait(v_full(s), (it / ST) & 1, abort, kErrVFull, status)) { ok = false; break; }
              v_ready = true;
            }
            if (!mbar_wait(p_full(t), p_cnt[t] & 1, abort, kErrPFull, status)) { ok = false; break; }
            tc_fence_after();
            issue_pv(t, s, j == 0);
            if constexpr (SPLIT_PASS) issue_pv_lo(t, s);
            ++p_cnt[t];
            tc_commit(o_done(t));
            if (j + 1 < x.n_t[t]) {
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
          if (x.n_t[t] > 0) ++ofree_cnt[t];
        kv_it += nmax;
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
      RingTileGeo x;
      if (!ring_tile_geo(p, tile, BN, x) || !in_pass(x)) continue;
      const int nn = x.n_t[t];
      if (nn == 0) continue;  // this query tile lies past the half's end
      const int first = x.q0 + t * BM;
      const int key_lim = first + r + x.g.diag;  // step 0 only
      const float qd = (TR::FP8 && p.q_descale != nullptr) ? p.q_descale[x.w.kvh] : 1.0f;
      // score scale (log2 units) and V descale of step s: the descales of its source rank
      auto step_scales = [&](int s, float& sc, float& vs) {
        const int src = (p.rank - s + p.S) % p.S;
        sc = p.scale_log2 * qd;
        vs = 1.0f;
        if constexpr (TR::FP8) {
          if (p.k_descales != nullptr) sc *= p.k_descales[src * p.Hkv + x.w.kvh];
          if (p.v_descales != nullptr) vs = p.v_descales[src * p.Hkv + x.w.kvh];
        }
      };
      float scale, vscale;
      step_scales(0, scale, vscale);
      int step = 0;
      float m = kNegInf, l = 0.f;  // m: running max of the scaled scores (log2 units)

      // one K/V tile of the online softmax (SPLIT: its e4m3 P as two terms, fp8_p_to_tmem);
      // fo: O factor when the V descale changes with the step; false when a wait gave up
      auto softmax_tile = [&](int j, int kbase, int seg, float fo, auto split_tag) -> bool {
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

        const int seg_len = x.g.len(seg);
        const bool causal = seg == 0;
        const bool need_mask = (kbase + BN > seg_len) || (causal && kbase + BN - 1 > first + x.g.diag);
        if (need_mask) {
#pragma unroll
          for (int c = 0; c < BN / 32; ++c)
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              const int key = kbase + c * 32 + e;
              if (key >= seg_len || (causal && key > key_lim)) sr[c][e] = __float_as_uint(kNegInf);
            }
        }
        float mx4[4] = {kNegInf, kNegInf, kNegInf, kNegInf};
#pragma unroll
        for (int c = 0; c < BN / 32; ++c)
#pragma unroll
          for (int e = 0; e < 32; e += 2)
            mx4[c] = fmax3(mx4[c], __uint_as_float(sr[c][e]), __uint_as_float(sr[c][e + 1]));
        const float mx = fmax3(fmaxf(mx4[0], mx4[1]), mx4[2], mx4[3]) * scale;  // scale > 0
        const float m_new = fmaxf(m, mx);
        if (j == 0) {
          m = m_new;
        } else {
          const bool need = (m_new - m) > kRescaleThreshold;
          if (__any_sync(0xffffffffu, need) || fo != 1.0f) {  // fo is uniform in the CTA
            // PV_t(j-1) is complete: S_t(j) was issued after it and has completed.
            const float f = need ? ex2_approx(m - m_new) : 1.0f;
            if (need) { l *= f; m = m_new; }
            const uint64_t f2 = f2pack(f * fo, f * fo);
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
        const float neg_m = (m == kNegInf) ? 0.f : -m;
        const uint64_t negm2 = f2pack(neg_m, neg_m);
        const uint64_t scale2 = f2pack(scale, scale);
        uint64_t rs2[2] = {0ull, 0ull};
        if constexpr (TR::FP8) {
          rs2[0] = fp8_p_to_tmem<TR, SPLIT>(sr, scale2, negm2, t_lane + uint32_t(TR::tm_s(t)));
          tmem_wait_st();
          tc_fence_before();
          mbar_arrive(p_full(t));
        } else {
          // P in 64-key halves: exps of a half are kept (as fp32 bits, in place of S) for the
          // row sum, which is added up after P has been handed to the MMA warp
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
          }
          tmem_wait_st();
          tc_fence_before();
          mbar_arrive(p_full(t));
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
      // the tile walk of this CTA tile (SPLIT_PASS: every tile's P split in two)
      auto walk = [&](auto split_tag) -> bool {
        SegCursor cur;
        cur.start(x.g, BN);
        for (int j = 0; j < nn; ++j) {
          cur.seek(x.g, j, BN);
          float fo = 1.0f;
          if (cur.s != step) {
            step = cur.s;
            float vs_new;
            step_scales(step, scale, vs_new);
            fo = vscale / vs_new;
            vscale = vs_new;
          }
          if (!softmax_tile(j, (j - cur.first) * BN, cur.s, fo, split_tag)) return false;
        }
        return true;
      };
      if (!walk(std::integral_constant<bool, SPLIT_PASS>{})) aborted = true;
      if (aborted) break;

      // ---------------------------------------------------------- epilogue of this tile
      pv_cnt += nn;
      {
        bool ok = mbar_wait(o_done(t), (pv_cnt - 1) & 1, abort, kErrODone, status);
        if (!__all_sync(0xffffffffu, ok)) { aborted = true; break; }
      }
      tc_fence_after();
      const bool valid = r < x.rows_t[t];
      const int64_t grow = int64_t(x.q_start) + first + r;
      const bool any_key = (m != kNegInf) && (l > 0.f);
      const float inv_l = any_key ? vscale / l : 0.f;  // O is in units of the last V descale
      uint8_t* orow = static_cast<uint8_t*>(p.out) + (grow * p.Hq + x.w.head) * int64_t(D) * 2;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        tmem_ld32(t_lane + uint32_t(TR::tm_o(t) + c * 32), o);
        tmem_wait_ld();
        reg_fence32(o);
        if (c == D / 32 - 1) {
          // all of O_t has been read: the next tile's PV_t may overwrite it
          tc_fence_before();
          mbar_arrive(o_free(t));
        }
        if (valid) {
          uint4* dst = reinterpret_cast<uint4*>(orow + c * 64);
#pragma unroll
          for (int v4 = 0; v4 < 4; ++v4) {
            uint32_t wd[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float f0 = __uint_as_float(o[v4 * 8 + 2 * i]) * inv_l;
              const float f1 = __uint_as_float(o[v4 * 8 + 2 * i + 1]) * inv_l;
              wd[i] = p.out_bf16 ? pack_bf16x2(f0, f1) : pack_f16x2(f0, f1);
            }
            dst[v4] = make_uint4(wd[0], wd[1], wd[2], wd[3]);
          }
        }
      }
      if (valid)
        p.lse[grow * p.Hq + x.w.head] = any_key ? (m + lg2_approx(l)) * kLn2 : kNegInf;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 9) tmem_dealloc(tmem, TR::TM_COLS);
}
