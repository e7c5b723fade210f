/*
 * dropkv_b200 -- C ABI of the B200-native DropKV prefill eviction path.
 *
 * The path scores every cached key position of every (sequence, KV head) by how
 * much dropping it would perturb the attention output of the last `window`
 * queries, max-pools the scores, protects the newest positions, keeps the top
 * `keep_len` positions per head and compacts their K/V rows.
 *
 * Conventions shared by every entry point:
 *   - All tensor pointers are CUDA device pointers on the current device.
 *   - K and V are contiguous [B, Hkv, Lk, D]; Q is [B, Hq, Lq, D] with arbitrary
 *     element strides (only its last `window` rows are read).  Q is tail-aligned:
 *     query row Lq-1 corresponds to key position Lk-1.
 *   - Query head h belongs to KV head h / (Hq / Hkv) (contiguous GQA groups).
 *   - `dtype` is one of DROPKV_DTYPE_*; Q, K and V share it.
 *   - `stream` is a cudaStream_t (NULL = legacy default stream).  Every call only
 *     enqueues work; nothing synchronises the host.
 *   - Scratch memory is passed in by the caller (`workspace`, at least the size the
 *     matching *_workspace_size function returns, 256-byte aligned).
 *   - Return value: DROPKV_OK or an error code; dropkv_last_error() returns a
 *     message for the calling host thread.  Kernels never trap.
 *
 * Reference interfaces replaced (paths inside the reference project):
 *   dropkv_scores          <- dropkv_triton.py:643-828  dropkv_scores_triton
 *   dropkv_select          <- dropkv_cache.py:462-477   max_pool1d + protect + topk + sort
 *   dropkv_gather          <- dropkv_cache.py:479-491   DropKVCache._gather_compressed
 *   dropkv_compress        <- dropkv_cache.py:355-491   _compute_keep_indices + _gather_compressed
 *   dropkv_compress_strided <- dropkv_cache.py:581-607  the same over in-place row buffers (no torch.cat)
 *   dropkv_compress_kv_strides <- dropkv_cache.py:355-491  the same over K/V views of any row-contiguous layout
 *   dropkv_compress_varlen <- dropkv_cache.py:355-491 and 470-473, 749-788: dropkv_compress over a
 *                             ragged batch in one call, keep_len per sequence evaluated on the device
 */
#ifndef DROPKV_B200_H
#define DROPKV_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define DROPKV_API __attribute__((visibility("default")))
#else
#define DROPKV_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum {
  DROPKV_DTYPE_F32 = 0,
  DROPKV_DTYPE_F16 = 1,
  DROPKV_DTYPE_BF16 = 2
};

enum {
  DROPKV_OK = 0,
  DROPKV_ERR_ARG = 1,         /* invalid shape, dtype, window, alignment ... */
  DROPKV_ERR_WORKSPACE = 2,   /* workspace pointer NULL / too small / misaligned */
  DROPKV_ERR_CUDA = 3,        /* a CUDA runtime call or launch failed */
  DROPKV_ERR_UNSUPPORTED = 4, /* valid request this build has no kernel for (e.g. D) */
  DROPKV_ERR_DEVICE = 5       /* a kernel reported a device-side status */
};

/* Round p to the input dtype before the weight (dropkv_triton.py:584-587). */
enum { DROPKV_ROUND_NONE = 0, DROPKV_ROUND_BF16 = 1, DROPKV_ROUND_F16 = 2 };

DROPKV_API const char* dropkv_version(void);
DROPKV_API const char* dropkv_last_error(void);

/* Number of kernel launches this library has issued in this process (all
 * devices, all threads); lets a harness count the launches of a timed region. */
DROPKV_API uint64_t dropkv_launch_count(void);

/* Scratch bytes dropkv_scores needs for this problem on the current device.
 * Replaces the intermediates allocated at dropkv_triton.py:736-769. */
DROPKV_API size_t dropkv_scores_workspace_size(int B, int Hq, int Hkv, int Lk, int D, int window);

/* scores[B, Hkv, Lk] (fp32) = DropKV eviction scores.
 * Replaces dropkv_triton.py:643-828 (dropkv_scores_triton: Q window slice,
 * Kernel A / split-A + C, Kernel B).  `window` is the number of query rows used
 * (1 <= window <= Lq <= Lk), `eps` the weight constant, `round_p` one of
 * DROPKV_ROUND_*.  q_s* are Q's element strides. */
DROPKV_API int dropkv_scores(const void* q, int64_t q_sb, int64_t q_sh, int64_t q_ss, int64_t q_sd, int Lq,
                  const void* k, const void* v, int dtype, int B, int Hq, int Hkv, int Lk, int D,
                  int window, float eps, int round_p, float* scores,
                  void* workspace, size_t workspace_bytes, void* stream);

/* Which scorer serves this problem: 2 = fused tensor-core kernel (tcgen05 +
 * TMA; bf16/fp16, D in {64,128}, g*window <= 64), 1 = CUDA-core split-K kernels
 * (every other supported problem).  0 for invalid sizes. */
DROPKV_API int dropkv_scorer_for(int dtype, int B, int Hq, int Hkv, int Lk, int D, int window);

/* Process-wide scorer selection: 0 = automatic (default), 1 = always the
 * CUDA-core kernels, 2 = always the tensor-core kernel (calls it does not cover
 * fail with DROPKV_ERR_UNSUPPORTED).  For testing one path against the other. */
DROPKV_API int dropkv_set_scorer(int mode);

/* Test hook for the tensor-core scorer's failure path (process-wide, for the
 * launches that follow).  wait_limit_ns: how long a wait on another warp role or
 * another CTA may last before the kernel gives up, records a non-zero status word
 * and runs to its end without further waits (0 = the default, 1 s).
 * block_group_barrier != 0: each launch starts head 0's first group barrier
 * below zero, so that barrier cannot complete and its wait runs out.  Nothing
 * faults or traps: the launch ends with the status set, the call returns
 * DROPKV_OK, and the next launch (hook off) is unaffected.  No counterpart in the
 * reference. */
DROPKV_API int dropkv_test_scorer_waits(uint64_t wait_limit_ns, int block_group_barrier);

/* Byte offset, inside a dropkv_scores / dropkv_compress workspace, of the int32
 * device status word the tensor-core scorer writes (0 = every bounded wait
 * completed; non-zero = a wait timed out and the results are invalid).
 * (size_t)-1 when the problem runs on the CUDA-core kernels. */
DROPKV_API size_t dropkv_scores_status_offset(int dtype, int B, int Hq, int Hkv, int Lk, int D, int window);

/* Size of the static device buffer dropkv_scores_static works in (16 MiB per
 * device).  It covers one 128K-token Llama-3.1-8B layer (8 KV heads, 32 window
 * rows, D = 128: about 10 MB of split partials on the tensor-core scorer). */
#define DROPKV_STATIC_SCRATCH_BYTES (16u << 20)

/* dropkv_scores without a workspace argument and without allocating anything:
 * no cudaMalloc / cudaFree and no allocating library call.  For callers that may
 * not allocate device memory when they score -- an engine that reserves all of
 * its device memory up front in its own pool, or a host thread that must not
 * enter an allocator -- and so cannot provide the scratch dropkv_scores takes.
 * The scratch is a DROPKV_STATIC_SCRATCH_BYTES buffer compiled into the library
 * (one per device).  Arguments, results and errors as dropkv_scores, plus:
 *   - the call is accepted when the scratch the scorer for this dtype needs fits
 *     the buffer (dropkv_scores_workspace_size, the larger of the bf16 and fp32
 *     needs, at most DROPKV_STATIC_SCRATCH_BYTES guarantees that); otherwise it
 *     returns DROPKV_ERR_WORKSPACE with a message naming both sizes, and
 *     launches nothing;
 *   - the first call on each device looks the buffer's address up (and, like
 *     every first scoring call, sets kernel attributes): make that first call
 *     before any stream capture;
 *   - the part of the scratch that must be zero when the kernels start (group
 *     barrier counters, status word) is zeroed by the call itself on `stream`
 *     (cudaMemsetAsync) before each launch; the caller initialises nothing;
 *   - all calls on one device share the buffer: two calls whose work can overlap
 *     on the device (unordered streams, or several host threads) race on it and
 *     give wrong scores.  Order them (one stream, or events);
 *   - the device status word of the call (non-zero: a bounded wait in the
 *     tensor-core scorer timed out and the scores are invalid) lives in the
 *     buffer; dropkv_scores_static_status copies it out.
 * No counterpart in the reference. */
DROPKV_API int dropkv_scores_static(const void* q, int64_t q_sb, int64_t q_sh, int64_t q_ss, int64_t q_sd,
                                    int Lq, const void* k, const void* v, int dtype, int B, int Hq, int Hkv,
                                    int Lk, int D, int window, float eps, int round_p, float* scores,
                                    void* stream);

/* Copies, by an asynchronous copy on `stream`, the int32 device status word of
 * the last dropkv_scores_static call on the current device for this problem
 * (same dtype and sizes) to *status_out: device memory, or host memory the
 * device can address (pinned).  0 = every bounded wait completed; problems on
 * the CUDA-core scorer, which has no bounded waits, always read 0.  Enqueue it
 * on the stream of that call, after it; allocates nothing.
 * No counterpart in the reference. */
DROPKV_API int dropkv_scores_static_status(int dtype, int B, int Hq, int Hkv, int Lk, int D, int window,
                                           int* status_out, void* stream);

/* Scratch bytes dropkv_select needs. */
DROPKV_API size_t dropkv_select_workspace_size(int B, int Hkv, int Lk);

/* keep_idx[B, Hkv, keep_len] (int64, ascending) = top-keep_len positions of
 * max_pool1d(scores, kernel_size, pad kernel_size/2, stride 1) after the last
 * min(protect_window, Lk) positions are set to amax + 1.  Ties are broken towards
 * the lower index.  Replaces dropkv_cache.py:464-475. */
DROPKV_API int dropkv_select(const float* scores, int B, int Hkv, int Lk, int kernel_size, int protect_window,
                  int keep_len, int64_t* keep_idx, void* workspace, size_t workspace_bytes,
                  void* stream);

/* k_out/v_out[B, Hkv, keep_len, D] = rows keep_idx of K/V (bit-exact copy).
 * elem_bytes is 2 or 4.  Replaces dropkv_cache.py:479-491. */
DROPKV_API int dropkv_gather(const void* k, const void* v, int elem_bytes, int B, int Hkv, int Lk, int D,
                  const int64_t* keep_idx, int keep_len, void* k_out, void* v_out, void* stream);

/* Scratch bytes dropkv_compress needs. */
DROPKV_API size_t dropkv_compress_workspace_size(int B, int Hq, int Hkv, int Lk, int D, int window);

/* The whole path in one call: scores -> pool/protect -> top-k -> sort -> gather.
 * scores_out may be NULL (scores then live in the workspace).  Replaces the
 * composition at dropkv_cache.py:355-491 (_compute_keep_indices followed by
 * _gather_compressed). */
DROPKV_API int dropkv_compress(const void* q, int64_t q_sb, int64_t q_sh, int64_t q_ss, int64_t q_sd, int Lq,
                    const void* k, const void* v, int dtype, int B, int Hq, int Hkv, int Lk, int D,
                    int window, float eps, int round_p, int kernel_size, int protect_window,
                    int keep_len, float* scores_out, int64_t* keep_idx, void* k_out, void* v_out,
                    void* workspace, size_t workspace_bytes, void* stream);

/* dropkv_compress for K/V kept in preallocated per-layer row buffers: K and V
 * are [B, Hkv, capacity, D] with kv_head_stride = capacity * D elements between
 * consecutive (b, kv head) rows (>= Lk * D, a multiple of 8); their first Lk rows
 * are scored.  The kept rows go to k_out / v_out laid out the same way with
 * out_head_stride elements between heads (>= keep_len * D, a multiple of 8; may be
 * the other buffer of a ping-pong pair, not the input itself).  Lets a chunked
 * prefill append each chunk in place and compact in place instead of copying the
 * whole cache per chunk as the reference's storage does
 * (dropkv_cache.py:581-607: torch.cat of stored + new K/V before every
 * eviction).  Results equal dropkv_compress on the same rows. */
DROPKV_API int dropkv_compress_strided(const void* q, int64_t q_sb, int64_t q_sh, int64_t q_ss, int64_t q_sd,
                                       int Lq, const void* k, const void* v, int64_t kv_head_stride, int dtype,
                                       int B, int Hq, int Hkv, int Lk, int D, int window, float eps, int round_p,
                                       int kernel_size, int protect_window, int keep_len, float* scores_out,
                                       int64_t* keep_idx, void* k_out, void* v_out, int64_t out_head_stride,
                                       void* workspace, size_t workspace_bytes, void* stream);

/* One sequence of a ragged batch for dropkv_compress_varlen. */
typedef struct dropkv_varlen_seq {
  const void* q;                    /* Q [B, Hq, Lq, D] with the element strides below */
  int64_t q_sb, q_sh, q_ss, q_sd;
  int Lq;
  int B;                            /* (b) rows of this sequence, e.g. its layers stacked */
  int Lk;                           /* keys */
  int cap;                          /* rows of room per (b, KV head) in the outputs, 1 <= cap <= Lk */
  const void* k;                    /* K, V [B, Hkv, Lk, D], contiguous */
  const void* v;
  int64_t* keep_idx;                /* [B, Hkv, cap] */
  void* k_out;                      /* [B, Hkv, cap, D] */
  void* v_out;
} dropkv_varlen_seq;

#define DROPKV_VARLEN_MAX_SEQS 32

DROPKV_API size_t dropkv_compress_varlen_workspace_size(int n_seq, const dropkv_varlen_seq* seqs, int Hq, int Hkv,
                                                        int D, int window);

/* dropkv_compress over a ragged batch of n_seq <= DROPKV_VARLEN_MAX_SEQS
 * sequences (host array `seqs`) in one call: each sequence is scored from its
 * last min(window, Lq) query rows (one scorer launch per sequence), then one
 * selection launch and one gather launch cover every (sequence, b, KV head) row.
 * keep_len of sequence s is evaluated on the device by the reference's rule
 * (dropkv_cache.py:470-473) and written to keep_len_out[s] (int32, device):
 *   min(Lk, max(int(keep_ratio * base), keep_window, 1)), base = total_tokens[s]
 *   if total_tokens (int64, device, may be NULL) else Lk, then
 *   min(max_keep_len[s]) if max_keep_len (int64, device, may be NULL; a negative
 *   entry sets no cap), and at most cap.
 * total_tokens / max_keep_len carry the seen-token count and the KV budget of the
 * reference's chunked-prefill policies (dropkv_cache.py:749-788) per sequence.
 * keep_idx / k_out / v_out rows past keep_len_out[s] are left untouched. The
 * first 4 bytes of the workspace receive the OR of the tensor-core scorer's
 * status words (non-zero: a bounded wait gave up). Kept sets equal those of
 * dropkv_compress per sequence with the same keep_len. */
DROPKV_API int dropkv_compress_varlen(int n_seq, const dropkv_varlen_seq* seqs, int dtype, int Hq, int Hkv, int D,
                                      int window, float eps, int round_p, int kernel_size, int protect_window,
                                      double keep_ratio, int keep_window, const int64_t* total_tokens,
                                      const int64_t* max_keep_len, int32_t* keep_len_out, void* workspace,
                                      size_t workspace_bytes, void* stream);

/* dropkv_compress over K and V of any layout whose rows of D elements are
 * contiguous: element strides kv_sb (sequence), kv_sh (KV head) and kv_ss (key),
 * each a multiple of 16 bytes, e.g. the [B, L, Hkv, D] projections that a model's
 * attention hands to DropKVCache.update as [B, Hkv, L, D] views
 * (dropkv_cache.py:493-622 receive them; the reference's torch ops read any
 * strides). Served by the tensor-core scorer (bf16/fp16, D 64/128, M <= 64);
 * other problems need packed rows and get DROPKV_ERR_UNSUPPORTED. Outputs as
 * dropkv_compress (K_c, V_c contiguous [B, Hkv, keep_len, D]); workspace:
 * dropkv_compress_workspace_size. */
DROPKV_API int dropkv_compress_kv_strides(const void* q, int64_t q_sb, int64_t q_sh, int64_t q_ss, int64_t q_sd,
                                          int Lq, const void* k, const void* v, int64_t kv_sb, int64_t kv_sh,
                                          int64_t kv_ss, int dtype, int B, int Hq, int Hkv, int Lk, int D,
                                          int window, float eps, int round_p, int kernel_size, int protect_window,
                                          int keep_len, float* scores_out, int64_t* keep_idx, void* k_out,
                                          void* v_out, void* workspace, size_t workspace_bytes, void* stream);

/* Appends `rows` rows per (b, kv head) of K and V (src: [BH, rows, D] with
 * src_head_stride elements between heads) at row dst_row of row buffers with
 * dst_head_stride elements between heads: one pitched device copy per tensor.
 * No counterpart in the reference, which concatenates the stored cache and the
 * new tokens into new tensors instead (dropkv_cache.py:581-617). */
DROPKV_API int dropkv_append_rows(void* k_dst, void* v_dst, int64_t dst_head_stride, int dst_row,
                                  const void* k_src, const void* v_src, int64_t src_head_stride, int rows,
                                  int D, int elem_bytes, int BH, void* stream);

/* Decode attention over the (compressed) cache: out[b, h, i, :] =
 * softmax(scale * q[b, h, i, :] . K[b, h / (Hq / Hkv), j, :]) V[b, h / (Hq / Hkv), j, :]
 * over the keys j <= L - Lq + i (the Lq query rows tail-aligned to the L keys).
 * Replaces the attention the model runs over the K/V that DropKVCache.update
 * returns (dropkv_cache.py:609-617 append the decode token to the compressed
 * cache; the model's SDPA attends over it). k/v: rows of D contiguous elements,
 * kv_sh elements between KV heads and kv_sb between sequences (a row buffer with
 * spare capacity is read in place), 16-byte aligned rows. bf16 or fp16, D 64 or
 * 128; out [B, Hq, Lq, D] contiguous in the input dtype. The workspace must be
 * zero-filled before its first use; every call leaves it ready for the next. */
DROPKV_API size_t dropkv_decode_attention_workspace_size(int B, int Hq, int Hkv, int Lq, int L, int D);
DROPKV_API int dropkv_decode_attention(const void* q, int64_t q_sb, int64_t q_sh, int64_t q_ss, int64_t q_sd,
                                       int Lq, const void* k, const void* v, int64_t kv_sb, int64_t kv_sh,
                                       int dtype, int B, int Hq, int Hkv, int L, int D, float scale, void* out,
                                       void* workspace, size_t workspace_bytes, void* stream);

/* dropkv_decode_attention fused with the append of the decode token(s): the
 * n_new rows of k_new / v_new ([B, Hkv, n_new, D], element strides new_sb, new_sh,
 * rows of D contiguous) are stored into the row buffers k / v at rows
 * [pos, pos + n_new) and attended over together with rows [0, pos), in one launch
 * (what dropkv_append_rows followed by dropkv_decode_attention over pos + n_new
 * keys give, bit for bit). Replaces the decode-time cache append and attention
 * (dropkv_cache.py:609-617 concatenate the token, the model's SDPA attends).
 * Workspace: dropkv_decode_attention_workspace_size(B, Hq, Hkv, Lq, pos + n_new, D). */
DROPKV_API int dropkv_decode_append_attention(const void* q, int64_t q_sb, int64_t q_sh, int64_t q_ss, int64_t q_sd,
                                              int Lq, const void* k_new, const void* v_new, int64_t new_sb,
                                              int64_t new_sh, int n_new, void* k, void* v, int64_t kv_sb,
                                              int64_t kv_sh, int pos, int dtype, int B, int Hq, int Hkv, int D,
                                              float scale, void* out, void* workspace, size_t workspace_bytes,
                                              void* stream);

/* Diagnostic: one 128-row tile through a tcgen05 MMA form used by the fused
 * scorer (mode 0: out[128][n] = A[128][128] B[n][128]^T with A loaded by TMA;
 * mode 1: out[128][n] = A[128][128]^T B[n][128]^T with A read MN-major; modes 2/3:
 * the same with 64-wide A rows; mode 4: mode 1 with B stored MN-major, n = 16/32/64;
 * mode 5: mode 4 with B split into two MN-major atoms of n/2 columns, n = 32/64/128).  a, b bf16 row-major; out fp32 [128][n];
 * *status (device int, zeroed by the caller) becomes non-zero if a wait timed out.
 * No counterpart in the reference: a hardware check of this library's building
 * blocks. */
DROPKV_API int dropkv_selftest_tcgen05(int mode, const void* a, const void* b, int n, float* out,
                                       int* status, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* DROPKV_B200_H */
