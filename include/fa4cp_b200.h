/*
 * fa4cp_b200 -- C ABI of the B200 (sm_100a) zig-zag ring-attention hot path.
 *
 * The reference (hxy0118/fa4-cp, package `fa4_ring`) is pure Python: its GPU work
 * goes through third-party Python-callable kernels (FlashAttention-4
 * `_flash_attn_fwd`, flashinfer `cascade.merge_state_in_place` / `merge_states`)
 * and ATen indexing.  Each entry point below replaces one of those call sites;
 * the citation names the reference file:line of the call it stands in for.
 *
 * Conventions (all entry points):
 *   - every pointer argument is a DEVICE pointer unless documented as host;
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream);
 *   - tensors are contiguous, row-major: Q/O [T, H, D], K/V [T, Hkv, D], LSE [T, H];
 *   - LSE is float32 natural log, layout [T, H];
 *   - nothing is allocated; every launch is asynchronous on `stream`;
 *   - return 0 on success or a negative FA4CP_ERR_* code; fa4cp_last_error()
 *     returns a description of the most recent failure of the calling thread.
 */
#ifndef FA4CP_B200_H_
#define FA4CP_B200_H_

#include <stdint.h>

#if defined(__GNUC__)
#define FA4CP_API __attribute__((visibility("default")))
#else
#define FA4CP_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define FA4CP_OK 0
#define FA4CP_ERR_INVALID (-1)     /* bad argument (maps to AssertionError/ValueError) */
#define FA4CP_ERR_UNSUPPORTED (-2) /* valid but not implemented (head_dim, dtype, ...) */
#define FA4CP_ERR_CUDA (-3)        /* CUDA runtime/driver error */
#define FA4CP_ERR_DEVICE (-4)      /* a kernel gave up a bounded wait (see device status) */

/* element types */
#define FA4CP_DTYPE_F16 0
#define FA4CP_DTYPE_BF16 1
#define FA4CP_DTYPE_F32 2
#define FA4CP_DTYPE_E4M3 3

/* ring step patterns (fa4_ring/ring_attention.py:11-16) */
#define FA4CP_PATTERN_VARLEN 0   /* q rows [cu_q[j],cu_q[j+1]) x k rows [cu_k[j],cu_k[j+1]) */
#define FA4CP_PATTERN_FRONT_KV 1 /* q rows [cu[j],cu[j+1]) x k rows [cu[j], mid_j)  (step <= rank) */
#define FA4CP_PATTERN_BACK_Q 2   /* q rows [mid_j,cu[j+1]) x k rows [cu[j],cu[j+1]) (step > rank) */

/* Library version (major*10000 + minor*100 + patch). */
FA4CP_API int fa4cp_version(void);

/* Text of the calling thread's most recent error ("" if none). */
FA4CP_API const char* fa4cp_last_error(void);

/*
 * Device status word written by kernels that gave up a bounded wait (0 = ok).
 * Synchronises the current device.  If `clear` != 0 the word is reset to 0.
 */
FA4CP_API int fa4cp_device_status(int32_t* status, int32_t clear);

/*
 * Self-test of the kernels' failure handling, with no GPU fault: launches one small
 * causal attention (q/k/v [seqlen, 1, 128] bf16, out bf16, lse float32, cu = {0, seqlen})
 * whose copy of K tile 0 is withheld, so the consumer's bounded mbarrier wait (~2 s) must
 * give up.  The kernel then records a status code, lets its issued copies and MMAs
 * finish, frees its tensor memory and returns.  Synchronises `stream`, writes the status
 * word the kernel recorded to *status_out (non-zero expected) and clears it.
 * No counterpart in the reference (its kernels come from FA4 and have no such path).
 */
FA4CP_API int fa4cp_selftest_wait_expiry(const void* q, const void* k, const void* v, void* out,
                                         float* lse, const int32_t* cu, int32_t seqlen,
                                         int32_t* status_out, void* stream);

/*
 * Variable-length attention forward returning out + LSE; also the three zig-zag
 * ring step patterns with in-place row addressing (no gathers).
 *
 * Replaces: fa4_ring/fa4_backend.py:58-123 (FA4 `_flash_attn_fwd` call :106-120,
 * LSE transpose :121-122) and the step-pattern row selections of
 * fa4_ring/ring_attention.py:109-166 (index_select/index_copy_ staging).
 *
 *   q            [total_q, Hq, D]   f16 | bf16 | e4m3
 *   k, v         [total_k, Hkv, D]  same dtype as q
 *   out          [total_q, Hq, D]   out_dtype (f16 | bf16; bf16 for e4m3 inputs)
 *   lse          [total_q, Hq]      float32, natural log
 *   cu_q         int32 [nseq+1]     query sequence boundaries (local cu for patterns 1,2)
 *   cu_k         int32 [nseq+1]     key boundaries (pattern VARLEN only; may equal cu_q)
 *   max_seqlen_q upper bound on any cu_q[j+1]-cu_q[j] (sizes the grid)
 *   pattern      FA4CP_PATTERN_*
 *   causal       1: key j visible to query i iff j <= i + (Tk - Tq)  (Tq == Tk: tril)
 *   softmax_scale  multiplier of q.k (the caller passes 1/sqrt(D) for the default)
 *   q/k/v_descale  NULL or float32 [Hkv] (e4m3 only): scores *= qd*kd, out *= vd
 *   accumulate   0: write out/lse of the covered rows;
 *                1: merge this partial into (out, lse) in place, online-softmax,
 *                   natural-log (the incremental merge of fa4_ring/merge.py:45-64 fused
 *                   into the epilogue); rows not covered are left untouched.
 * Supported: head_dim 64, 128 or 256 (f16/bf16), 128 (e4m3); Hq % Hkv == 0.
 */
FA4CP_API int fa4cp_attn_fwd(const void* q, const void* k, const void* v, void* out, float* lse,
                   const int32_t* cu_q, const int32_t* cu_k, int32_t nseq, int32_t max_seqlen_q,
                   int64_t total_q, int64_t total_k, int32_t num_heads_q, int32_t num_heads_kv,
                   int32_t head_dim, int32_t in_dtype, int32_t out_dtype, int32_t pattern,
                   int32_t causal, float softmax_scale, const float* q_descale,
                   const float* k_descale, const float* v_descale, int32_t accumulate,
                   void* stream);

/*
 * Attention over a PAGED K/V cache (variable-length, causal or not): fa4cp_attn_fwd's
 * VARLEN pattern with K/V rows looked up through a block table instead of contiguous rows.
 *   k_pages, v_pages  [num_pages, page_size, Hkv, D] page pools (dtype as q)
 *   block_table       int32 [nseq, max_pages_per_seq]: physical page of each logical page
 *   page_size         a multiple of 128 (a K/V tile never straddles two pages)
 *   cu_k              int32 [nseq+1] LOGICAL cumulative K/V lengths (sequence j has
 *                     cu_k[j+1]-cu_k[j] <= max_pages_per_seq * page_size keys)
 * Other arguments as fa4cp_attn_fwd (no accumulate).  Page indices are read on the device and
 * not validated; one outside [0, num_pages) reads zeros.  head_dim 64 / 128 (f16, bf16), 128
 * (e4m3).  No counterpart in the reference, whose rotated K/V is contiguous
 * (its README's "no paged KV" limitation, README.md:139-141).
 */
FA4CP_API int fa4cp_attn_fwd_paged(const void* q, const void* k_pages, const void* v_pages,
                                   const int32_t* block_table, int32_t page_size,
                                   int32_t num_pages, int32_t max_pages_per_seq, void* out,
                                   float* lse, const int32_t* cu_q, const int32_t* cu_k,
                                   int32_t nseq, int32_t max_seqlen_q, int64_t total_q,
                                   int32_t num_heads_q, int32_t num_heads_kv, int32_t head_dim,
                                   int32_t in_dtype, int32_t out_dtype, int32_t causal,
                                   float softmax_scale, const float* q_descale,
                                   const float* k_descale, const float* v_descale, void* stream);

/*
 * Attention with a bf16 query and e4m3 keys/values (mixed precision, e.g. FP8 KV with a
 * bf16 Q).  One tcgen05 MMA takes a single operand type, so K and V are first
 * dequantised (value x per-kv-head descale) into `workspace` as bf16 and attended by the
 * bf16 kernel.  Arguments as fa4cp_attn_fwd (out/lse in the query dtype / float32);
 * k_descale, v_descale: NULL or float32 [Hkv].
 *   workspace        device buffer of >= fa4cp_attn_kv8_workspace_bytes(total_k, Hkv, D)
 *                    bytes (scratch: contents are overwritten; calls sharing it must not
 *                    overlap on the GPU).
 * Replaces: the FP8-KV path of fa4_ring/fa4_backend.py:99-120 (FA4 `k_descale`/`v_descale`
 * with a non-FP8 query) used by the cfg "bf16 Q, FP8 e4m3 KV" of the reference's ring.
 */
FA4CP_API int fa4cp_attn_fwd_kv8(const void* q, const void* k8, const void* v8, void* out,
                                 float* lse, const int32_t* cu_q, const int32_t* cu_k,
                                 int32_t nseq, int32_t max_seqlen_q, int64_t total_q,
                                 int64_t total_k, int32_t num_heads_q, int32_t num_heads_kv,
                                 int32_t head_dim, int32_t q_dtype, int32_t pattern,
                                 int32_t causal, float softmax_scale, const float* k_descale,
                                 const float* v_descale, int32_t accumulate, void* workspace,
                                 int64_t workspace_bytes, void* stream);

/*
 * fa4cp_attn_fwd_kv8 without a workspace argument, for callers that cannot allocate
 * device memory when they call (an engine whose memory is already reserved for its own
 * pools, a caller that must not risk the synchronisation of cudaMalloc/cudaFree, or a
 * binding that holds only the tensors it was given).  The dequantised K/V go to a fixed
 * 32 MiB scratch array compiled into the library, so nothing is allocated.
 * No counterpart in the reference (its FA4 call allocates internally).
 *   limit: total_k * num_heads_kv * head_dim <= 8,388,608 (K and V in bf16 fill the 32 MiB);
 *          larger calls return FA4CP_ERR_INVALID;
 *   every GPU that loads this part of the library holds the 32 MiB until process exit;
 *   all calls on a device share the array (it keeps the last call's contents; nothing in
 *   it needs to start at zero); calls that overlap on the GPU race and must be serialised;
 *   the first call on a device looks up the array's device address (cudaGetSymbolAddress)
 *   and should come before any stream capture.
 * Other arguments as fa4cp_attn_fwd_kv8.
 */
FA4CP_API int fa4cp_attn_fwd_kv8_noalloc(const void* q, const void* k8, const void* v8, void* out,
                                         float* lse, const int32_t* cu_q, const int32_t* cu_k,
                                         int32_t nseq, int32_t max_seqlen_q, int64_t total_q,
                                         int64_t total_k, int32_t num_heads_q,
                                         int32_t num_heads_kv, int32_t head_dim, int32_t q_dtype,
                                         int32_t pattern, int32_t causal, float softmax_scale,
                                         const float* k_descale, const float* v_descale,
                                         int32_t accumulate, void* stream);

/* Workspace bytes fa4cp_attn_fwd_kv8 needs (2 * total_k * Hkv * D * 2), or -1 on bad input. */
FA4CP_API int64_t fa4cp_attn_kv8_workspace_bytes(int64_t total_k, int32_t num_heads_kv,
                                                 int32_t head_dim);

/*
 * e4m3 -> bf16 dequantisation: out = x * descale[head], x [rows, heads, dim] (dim % 16 == 0).
 * Replaces: the dequantised-KV path FA4 runs internally for descaled FP8 inputs.
 */
FA4CP_API int fa4cp_dequant_e4m3(const void* x, const float* descale, void* out, int64_t rows,
                                 int32_t heads, int32_t dim, void* stream);

/*
 * Per-tensor e4m3 quantisation of n elements (f16 | bf16 | f32): *scale = amax / 448
 * (1 if the tensor is all zero), out = satfinite(x / *scale) as e4m3.  `scale` is a device
 * float written by the call.  This is the per-rank quantisation the FP8 configs prescribe
 * before the ring (each rank's K/V descales are then all-gathered, indexed by source rank).
 */
FA4CP_API int fa4cp_quantize_e4m3(const void* x, int32_t dtype, int64_t n, void* out,
                                  float* scale, void* stream);

/*
 * In-place 2-way LSE merge: (v, s) <- merge((v, s), (v_other, s_other)).
 * Replaces: flashinfer `cascade.merge_state_in_place` as called by
 * fa4_ring/merge.py:31-36,60 (with natural-log LSE, fa4_ring/merge.py:17-18).
 *   v, v_other [num_rows, num_heads, head_dim] dtype (f16 | bf16 | f32); s, s_other [num_rows, num_heads]
 * Rows where s_other is -inf are left unchanged; head_dim % 8 == 0 (f16/bf16), % 4 (f32).
 */
FA4CP_API int fa4cp_merge_state_inplace(void* v, float* s, const void* v_other, const float* s_other,
                              int64_t num_rows, int32_t num_heads, int32_t head_dim, int32_t dtype,
                              void* stream);

/*
 * k-way LSE merge of `num_states` partials read through pointer arrays (no stack copy).
 * Replaces: flashinfer `cascade.merge_states` after torch.stack, fa4_ring/merge.py:39-42,83-85.
 *   v_ptrs, s_ptrs  HOST arrays of `num_states` device pointers (1 <= num_states <= 32)
 *   v_out [num_rows, num_heads, head_dim] dtype; s_out [num_rows, num_heads] float32 (may be NULL)
 */
FA4CP_API int fa4cp_merge_states(const void* const* v_ptrs, const float* const* s_ptrs, int32_t num_states,
                       void* v_out, float* s_out, int64_t num_rows, int32_t num_heads,
                       int32_t head_dim, int32_t dtype, void* stream);

/*
 * Fill a float32 buffer with `value` (used to mark rows a partial does not cover
 * with LSE = -inf, as fa4_ring/ring_attention.py:162-163 does with torch.full).
 */
FA4CP_API int fa4cp_fill_f32(float* dst, int64_t n, float value, void* stream);

/*
 * Zig-zag gather: this rank's local shard of every packed sequence.
 * Replaces: fa4_ring/zigzag.py:31-39 (`zigzag_shard`) and :82-97 (`zigzag_shard_varlen`).
 *   x        [total_full, row_bytes] bytes; out [total_full / cp_size, row_bytes]
 *   full_cu  int32 [nseq+1] device boundaries of the FULL sequences, or NULL for a
 *            single sequence of total_full rows; every length must be divisible by
 *            2*cp_size (the caller validates; the kernel trusts it).
 */
FA4CP_API int fa4cp_zigzag_shard(const void* x, void* out, const int32_t* full_cu, int32_t nseq,
                       int64_t total_full, int32_t cp_rank, int32_t cp_size, int64_t row_bytes,
                       void* stream);

/*
 * Zig-zag scatter: stitch all ranks' local shards back into the full packed sequence.
 * Replaces: fa4_ring/zigzag.py:42-50 (`zigzag_unshard`) and the per-sequence stitching of
 * the reference's tests (tests/test_ring_correctness.py:29-36).
 *   shards   HOST array of `cp_size` device pointers, each [total_full / cp_size, row_bytes]
 *   out      [total_full, row_bytes]; full_cu as for fa4cp_zigzag_shard (NULL = one sequence)
 */
FA4CP_API int fa4cp_zigzag_unshard(const void* const* shards, void* out, const int32_t* full_cu,
                         int32_t nseq, int64_t total_full, int32_t cp_size, int64_t row_bytes,
                         void* stream);

/*
 * Device-side `get_half_index` (no host sync): int64 indices of the front (front=1)
 * or back (front=0) half of each packed local sequence.
 * Replaces: fa4_ring/zigzag.py:65-79 (`.tolist()` + Python loop of arange).
 *   cu int32 [nseq+1] (each length even); out_idx int64 [total / 2]
 */
FA4CP_API int fa4cp_half_index(const int32_t* cu, int32_t nseq, int64_t total, int32_t front,
                     int64_t* out_idx, void* stream);

/*
 * GDN context-parallel index metadata, on the device.
 * Replaces: the Python loops of fa4_ring/gdn_cp/metadata.py:48-96 (build_gdn_cp_metadata).
 *   full_cu int32 [nseq+1] natural-order boundaries (every length a multiple of 2*cp_size);
 *   restore_perm int64 [total] (or NULL): slot of natural token n in the rank-major
 *   all-gather of the local shards (rank r's part at r * total / cp_size);
 *   extract_idx int64 [total / cp_size] (or NULL): natural position of local token i of
 *   cp_rank.  The gathers themselves are fa4cp_zigzag_unshard (restore, with the shard
 *   pointers into the all-gather buffer) and fa4cp_zigzag_shard (extract).
 */
FA4CP_API int fa4cp_gdn_cp_indices(const int32_t* full_cu, int32_t nseq, int32_t cp_size,
                                   int32_t cp_rank, int64_t total, int64_t* restore_perm,
                                   int64_t* extract_idx, void* stream);

/*
 * local_cu[j] = full_cu[j] / cp_size for j in [0, nseq]  (the local cu_seqlens that
 * fa4_ring/zigzag.py:94-97 builds on the host).
 */
FA4CP_API int fa4cp_local_cu(const int32_t* full_cu, int32_t nseq, int32_t cp_size, int32_t* local_cu,
                   void* stream);

/*
 * Native ring executor (incremental merge mode): one call runs a rank's whole zig-zag ring
 * forward, every K/V hop as NCCL send/recv on the executor's high-priority comm stream and
 * every step's attention (fa4cp_attn_fwd / fa4cp_attn_fwd_kv8, with the in-epilogue merge) on
 * `stream`, ordered by CUDA events; the host never blocks.
 * Replaces: the per-step loop of fa4_ring/ring_attention.py:121-172 (torch.distributed
 * P2P + `_attn` + `merge_state_in_place` per step) with the reference's step schedule.
 *
 * Unlike the rest of this header, the ring handle owns resources: an NCCL communicator
 * (ncclCommInitRank; libnccl.so.2 found with dlopen), a comm stream and CUDA events.
 *
 * fa4cp_ring_unique_id: writes the 128-byte NCCL unique id (HOST buffer) that rank 0 makes
 *   and the caller broadcasts to the cp group.
 * fa4cp_ring_comm_init: collective over the cp group (every rank calls it with the same id,
 *   on the device it will run on); NCCL rank = cp rank; 1 <= nranks <= 64.  id NULL: no
 *   NCCL communicator (copy-engine transport only; not collective).  handle_out HOST int64.
 * fa4cp_ring_comm_destroy: waits for the comm stream and frees the communicator; call it on
 *   every rank before the process group is torn down.
 * fa4cp_ring_set_sm_reserve: SMs (0..64, default 8) the persistent attention grid leaves
 *   free during a ring call, so that the hop's NCCL kernel runs beside it.
 * fa4cp_ring_set_fused: mode 2 (default) runs the whole forward as one launch of the ring
 *   kernel (fa4cp_ring_attn_fused) for f16 / bf16 with D 64 or 128 and e4m3 with D 128
 *   (copy-engine transport or a single rank); mode 1 for f16 / bf16 only; mode 3 also at
 *   head_dim 256 (f16 / bf16, and bf16 q with e4m3 K/V through fa4cp_ring_attn_fused_mixed,
 *   the K/V converted to bf16 once per rank and pushed as such; the workspace of
 *   fa4cp_ring_attn_fwd then holds them); 0 keeps one attention launch per step.
 * fa4cp_ring_timing: time the next `max_launches` attention launches and hops (0 = off) with
 *   CUDA events; fa4cp_ring_timeline writes (start, end) pairs in ms relative to the first
 *   timed launch's start into HOST float arrays (attention launches and hops, in issue order,
 *   at most max_attn / max_hops pairs; counts to n_attn / n_hops); fa4cp_ring_timing_read
 *   waits for them and returns the launches' summed duration (HOST double, ms) and count
 *   (HOST int32), then starts over.
 * fa4cp_ring_attn_fwd:
 *   q [total, Hq, D], k/v [total, Hkv, D] this rank's zig-zag shards; out/lse [total, Hq(, D)]
 *   receive the merged result (out dtype: q's, bf16 for e4m3 q);
 *   kv_bufs (NCCL transport; NULL with the copy engine) >= 4 * total*Hkv*D*elem bytes,
 *   16-byte aligned (two receive slots of K and V); the copy engine needs
 *   total*Hkv*D*elem <= the kv_capacity of fa4cp_ring_ipc_alloc;
 *   cu int32 [nseq+1] local boundaries (even lengths), max_seqlen the longest local length;
 *   q_dtype/kv_dtype: equal (f16 | bf16 | e4m3), or bf16 q with e4m3 k/v (then `workspace`
 *   of fa4cp_attn_kv8_workspace_bytes(total, Hkv, D) bytes is required);
 *   k_descales/v_descales float32 [cp_size, Hkv] indexed by SOURCE rank (NULL for 16-bit
 *   k/v), q_descale float32 [Hkv] for e4m3 q.
 */
/*
 * Copy-engine transport of the ring executor (used when fa4cp_ring_ipc_open has run):
 * fa4cp_ring_ipc_alloc: (re)allocates this rank's receive area with cudaMalloc: a 4 KiB
 *   header (32-bit hop counters ARRIVED at byte 0 and FREED at byte 128), then nranks-1 K
 *   slots and nranks-1 V slots of kv_capacity bytes each (rounded up to 256; slot i of hop i+1
 *   of a call); writes its 64-byte CUDA IPC handle to ipc_out (HOST).  Synchronises the
 *   device; resets the hop count.
 * fa4cp_ring_ipc_open: maps the left and right neighbours' areas (HOST 64-byte handles; the
 *   same handle for both when nranks == 2).  fa4cp_ring_ipc_close unmaps them.
 * Every rank calls alloc, exchanges handles, and opens, with a barrier of the cp group
 * before freeing (close, barrier, alloc) and after opening; all ranks use the same capacity.
 * fa4cp_ring_ce_plan: the ordered operations one call issues (host only, no GPU needed),
 *   for hops g0+1 .. g0+nranks-1, with per-step attention launches (fused 0) or the
 *   persistent ring kernel (fused 1); returns the count (ops may be NULL to ask for it).
 */
typedef struct {
  int32_t stream; /* 0 caller's (compute), 1 K copy, 2 V copy, 3 release, 4 K copy 2, 5 V copy 2 */
  int32_t kind;   /* FA4CP_RING_OP_* */
  int64_t a, b, c;
} fa4cp_ring_op;
#define FA4CP_RING_OP_RECORD 0     /* record event a */
#define FA4CP_RING_OP_WAIT_EVENT 1 /* wait for event a's latest record */
#define FA4CP_RING_OP_WAIT_FLAG 2  /* wait until own counter a (0 arrived, 1 freed) >= b (cyclic) */
#define FA4CP_RING_OP_WRITE_FLAG 3 /* write counter b of peer a (0 right, 1 left) := c */
#define FA4CP_RING_OP_COPY 4       /* part a (0 K, 1 V): src b (-1 caller's, else own slot b)
                                      -> right neighbour's slot c */
#define FA4CP_RING_OP_ATTN 5       /* attention of step a on K/V b (-1 caller's, else own
                                      slot b) */
#define FA4CP_RING_OP_ATTN_FUSED 6 /* persistent ring kernel over a steps; before reading
                                      slot s-1 it waits for own ARRIVED >= b + s */
/* direct pushes (fa4cp_ring_set_direct): flags are 32-bit words of the receive area's header,
 * flag 2 + i = the arrival flag of slot i, flag 130 + d = FREED[d] (the release, by rank
 * rank + d, of the slot holding this rank's K/V); WAIT_FLAG a is such a flag index */
#define FA4CP_RING_OP_COPY_TO 7    /* part a (0 K, 1 V) of the caller's K/V -> slot c of rank
                                      rank + b */
#define FA4CP_RING_OP_WRITE_PEER 8 /* write flag b of rank rank + a := c */
#define FA4CP_RING_OP_ATTN_FUSED_SLOTS 9 /* persistent ring kernel over a steps on own slots
                                      c .. c+a-2; before reading slot c+s-1 it waits for that
                                      slot's arrival flag >= b */
FA4CP_API int fa4cp_ring_ipc_alloc(int64_t handle, int64_t kv_capacity, uint8_t* ipc_out);
FA4CP_API int fa4cp_ring_ipc_open(int64_t handle, const uint8_t* left_ipc,
                                  const uint8_t* right_ipc);
FA4CP_API int fa4cp_ring_ipc_close(int64_t handle);
FA4CP_API int fa4cp_ring_ce_plan(int32_t nranks, int32_t rank, int64_t g0, int32_t fused,
                                 fa4cp_ring_op* ops, int32_t capacity);

/*
 * Direct pushes (the copy-engine transport's default over NVSwitch; no counterpart in the
 * reference, whose rotation is a chain of P2P hops, fa4_ring/ring_attention.py:121-136):
 * at the start of call n every rank copies its own K/V straight into slot d-1 of rank
 * rank + d (d = 1 .. nranks-1, step order, two pairs of copy streams), then sets that slot's
 * arrival flag to n; the attention of step s waits for its slot's flag (the ring kernel does
 * so itself).  Slots come in two sets used by alternate calls, so a push of call n waits only
 * for the destination's release of call n-2: no call waits for the end of the previous one.
 * After its attention a rank sets FREED[s] := n at rank rank - s for every s.
 * fa4cp_ring_set_direct: on (1) or off (0, the chained hops of fa4cp_ring_ce_plan); call before
 *   fa4cp_ring_ipc_alloc (the area holds two slot sets when on).
 * fa4cp_ring_ipc_open_all: maps every peer's area (HOST: nranks x 64-byte handles, this rank's
 *   own included, indexed by rank); needed by direct pushes, enough for chained hops too.
 * fa4cp_ring_ce_direct_plan: the ordered operations of call number `call` (>= 1) with direct
 *   pushes (host only, no GPU needed); returns the count (ops may be NULL to ask for it).
 */
FA4CP_API int fa4cp_ring_set_direct(int64_t handle, int32_t on);
FA4CP_API int fa4cp_ring_ipc_open_all(int64_t handle, const uint8_t* ipc_handles);
FA4CP_API int fa4cp_ring_ce_direct_plan(int32_t nranks, int32_t rank, int64_t call, int32_t fused,
                                        fa4cp_ring_op* ops, int32_t capacity);

/*
 * Persistent ring kernel: the whole zig-zag ring forward of one rank in ONE launch.  Each
 * CTA owns two 128-row query tiles of one half (early / late) of one local sequence and one
 * query head, and walks the K/V of every step in order -- step 0 the local K/V (causal),
 * step s >= 1 the K/V of rank (rank - s) mod nranks in slot s-1 (front half when s <= rank;
 * all of it, for late-half rows only, when s > rank) -- carrying the online softmax across
 * steps, so out and lse are written once (no per-step merge).  Before its first read of
 * slot s-1 a CTA waits (bounded, ~10 s) until *arrived >= arrived_base + s; arrived NULL:
 * every slot is already filled.
 * Replaces: the whole step loop of fa4_ring/ring_attention.py:121-172 (attention per step
 * and the incremental merges of fa4_ring/merge.py:45-64).
 *   q [total, Hq, D], k/v [total, Hkv, D] local; slots_k / slots_v: slot i at
 *   slots_k + i * slot_stride bytes, each [total, Hkv, D] (the source's shard, same cu);
 *   out [total, Hq, D] (q dtype; bf16 for e4m3); lse [total, Hq] float32.  f16 / bf16 with
 *   D 64, 128 or 256, or e4m3 with D 128: then q_descale [Hkv] and k_descales / v_descales
 *   [nranks, Hkv] indexed by SOURCE rank (each may be NULL = 1); NULL for 16-bit inputs.
 *   D 256 runs one 128-row query tile per CTA (S and O of two tiles exceed TMEM).
 */
/*
 * Wall-time bound (ms, default 10000) of the ring kernel's wait for a hop counter; past it
 * the kernel records FA4CP status 0x10a (see fa4cp_device_status), lets its issued copies and
 * MMAs finish and returns.  Process-wide; applies to launches made after the call.
 */
FA4CP_API int fa4cp_ring_set_wait_timeout_ms(int32_t ms);

FA4CP_API int fa4cp_ring_attn_fused(const void* q, const void* k, const void* v,
                                    const void* slots_k, const void* slots_v,
                                    int64_t slot_stride, void* out, float* lse,
                                    const int32_t* cu, int32_t nseq, int32_t max_seqlen,
                                    int64_t total, int32_t num_heads_q, int32_t num_heads_kv,
                                    int32_t head_dim, int32_t dtype, float softmax_scale,
                                    const float* q_descale, const float* k_descales,
                                    const float* v_descales, int32_t nranks, int32_t rank,
                                    const uint32_t* arrived, uint32_t arrived_base,
                                    void* stream);
/*
 * fa4cp_ring_attn_fused_mixed: the ring kernel for a bf16 query with e4m3 K/V at head_dim 256
 * (the reference's bf16-Q x e4m3-K/V ring, fa4_ring/ring_attention.py:139-166, with the per-
 * source descales of fa4_ring/fa4_backend.py:99-120).  k, v and every slot hold the EXACT bf16
 * images of the e4m3 shards (fa4cp_dequant_e4m3 with a NULL descale: e4m3 -> bf16 is exact);
 * k_descales / v_descales [nranks, Hkv] by source rank (NULL = 1) are applied in fp32 inside the
 * kernel (score scale, output factor), so the result equals attention over the dequantised
 * K/V up to the kernel's bf16 P.  Slot stride and layout as fa4cp_ring_attn_fused (bf16
 * bytes).  out bf16 [total, Hq, 256]; lse float32 [total, Hq].
 */
FA4CP_API int fa4cp_ring_attn_fused_mixed(const void* q, const void* k, const void* v,
                                          const void* slots_k, const void* slots_v,
                                          int64_t slot_stride, void* out, float* lse,
                                          const int32_t* cu, int32_t nseq, int32_t max_seqlen,
                                          int64_t total, int32_t num_heads_q,
                                          int32_t num_heads_kv, int32_t head_dim,
                                          float softmax_scale, const float* k_descales,
                                          const float* v_descales, int32_t nranks, int32_t rank,
                                          const uint32_t* arrived, uint32_t arrived_base,
                                          void* stream);
/*
 * fa4cp_ring_attn_fused_remote: the same ring kernel over the remote steps 1 .. nranks-1 only,
 * merged into the (out, lse) already there -- the partial of step 0, the local K/V, causal, as
 * fa4cp_attn_fwd (VARLEN, causal) writes it.  f16 / bf16 only.  The executor's direct pushes run
 * a forward this way (no counterpart in the reference, whose merge is a separate pass,
 * fa4_ring/merge.py:45-64): the remote walk then starts once the first pushes have landed.
 */
FA4CP_API int fa4cp_ring_attn_fused_remote(const void* q, const void* k, const void* v,
                                           const void* slots_k, const void* slots_v,
                                           int64_t slot_stride, void* out, float* lse,
                                           const int32_t* cu, int32_t nseq, int32_t max_seqlen,
                                           int64_t total, int32_t num_heads_q,
                                           int32_t num_heads_kv, int32_t head_dim, int32_t dtype,
                                           float softmax_scale, int32_t nranks, int32_t rank,
                                           const uint32_t* arrived, uint32_t arrived_base,
                                           void* stream);

FA4CP_API int fa4cp_ring_unique_id(uint8_t* id_out);
FA4CP_API int fa4cp_ring_comm_init(const uint8_t* id, int32_t nranks, int32_t rank,
                                   int64_t* handle_out);
FA4CP_API int fa4cp_ring_comm_destroy(int64_t handle);
FA4CP_API int fa4cp_ring_set_sm_reserve(int64_t handle, int32_t sm_reserve);
FA4CP_API int fa4cp_ring_set_fused(int64_t handle, int32_t fused);
FA4CP_API int fa4cp_ring_timing(int64_t handle, int32_t max_launches);
FA4CP_API int fa4cp_ring_timeline(int64_t handle, float* attn_ms, int32_t max_attn,
                                  float* hop_ms, int32_t max_hops, int32_t* n_attn,
                                  int32_t* n_hops);
FA4CP_API int fa4cp_ring_timing_read(int64_t handle, double* total_ms, int32_t* launches);
FA4CP_API int fa4cp_ring_attn_fwd(int64_t handle, const void* q, const void* k, const void* v,
                                  void* kv_bufs, int64_t kv_bufs_bytes, void* out, float* lse,
                                  const int32_t* cu, int32_t nseq, int32_t max_seqlen,
                                  int64_t total, int32_t num_heads_q, int32_t num_heads_kv,
                                  int32_t head_dim, int32_t q_dtype, int32_t kv_dtype,
                                  float softmax_scale, const float* q_descale,
                                  const float* k_descales, const float* v_descales,
                                  void* workspace, int64_t workspace_bytes, void* stream);

/*
 * Attention BACKWARD of one ring step.  No counterpart in the reference, which is
 * forward-only (README.md:142: "forward-only (inference). No backward"); these are the
 * gradients of its forward (tests/test_algorithm_cpu.py:36-48) over the rows of the step
 * patterns of fa4_ring/ring_attention.py:109-166.  f16 / bf16, head_dim 64 or 128.
 *
 * fa4cp_attn_bwd_preprocess: delta[row, h] = sum_d dout * out   (float32 [total_q, Hq]);
 *   out, dout [total_q, Hq, D] in `dtype`, 4-byte aligned.
 * fa4cp_attn_bwd: ADDS one step's gradient contributions into float32 accumulators:
 *   dq_acc [total_q, Hq, D]  (added with atomics: every key tile adds into a query row)
 *   dk_acc, dv_acc [total_k, Hkv, D]  (read-add-write; a key row has one writer per launch)
 *   lse   float32 [total_q, Hq], natural log, of the FINAL output (so the steps' gradients
 *         add up); rows with lse -inf contribute nothing
 *   delta from fa4cp_attn_bwd_preprocess on the final output
 *   cu_q, cu_k, pattern, causal, softmax_scale: as fa4cp_attn_fwd (the step's rows)
 *   max_seqlen_k upper bound on any sequence's key count under `pattern` (sizes the grid:
 *         VARLEN max cu_k length; FRONT_KV half the max local length; BACK_Q the max)
 *   16-byte aligned q, k, v, dout and accumulators.  dq_acc's sums are fp32 atomics, so
 *   their rounding order (not the math) varies between runs.
 * fa4cp_convert_f32: dst (f16 | bf16 | f32) = src (float32), n elements.
 * fa4cp_add_f32: dst += src, n float32 elements, n % 4 == 0, 16-byte aligned.
 */
FA4CP_API int fa4cp_attn_bwd_preprocess(const void* out, const void* dout, float* delta,
                                        int64_t total_q, int32_t num_heads_q, int32_t head_dim,
                                        int32_t dtype, void* stream);
FA4CP_API int fa4cp_attn_bwd(const void* q, const void* k, const void* v, const void* dout,
                             const float* lse, const float* delta, float* dq_acc, float* dk_acc,
                             float* dv_acc, const int32_t* cu_q, const int32_t* cu_k,
                             int32_t nseq, int32_t max_seqlen_k, int64_t total_q, int64_t total_k,
                             int32_t num_heads_q, int32_t num_heads_kv, int32_t head_dim,
                             int32_t dtype, int32_t pattern, int32_t causal, float softmax_scale,
                             void* stream);
FA4CP_API int fa4cp_convert_f32(const float* src, void* dst, int64_t n, int32_t dst_dtype,
                                void* stream);
FA4CP_API int fa4cp_add_f32(float* dst, const float* src, int64_t n, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FA4CP_B200_H_ */
