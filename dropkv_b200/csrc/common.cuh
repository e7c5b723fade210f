// Shared device helpers and host-side plumbing for the dropkv_b200 kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <string>

#include "../../include/dropkv_b200.h"

namespace dropkv {

// ---------------------------------------------------------------------------
// Error reporting (per host thread)
// ---------------------------------------------------------------------------
void set_error(const char* fmt, ...);
int fail(int code, const char* fmt, ...);
int check_launch(const char* what, int launches = 1);

// ---------------------------------------------------------------------------
// Element conversion
// ---------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ float to_f(T x);
template <>
__device__ __forceinline__ float to_f<float>(float x) { return x; }
template <>
__device__ __forceinline__ float to_f<__half>(__half x) { return __half2float(x); }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }

// p rounded to the input dtype and widened back (torch's .to(dtype).float()).
__device__ __forceinline__ float round_p(float p, int mode) {
  if (mode == DROPKV_ROUND_BF16) return __bfloat162float(__float2bfloat16_rn(p));
  if (mode == DROPKV_ROUND_F16) return __half2float(__float2half_rn(p));
  return p;
}

// Float -> uint32 with unsigned order == float order; -0.0 maps like +0.0.
__device__ __forceinline__ uint32_t ordered_key(float f) {
  f = f + 0.0f;
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
// Programmatic dependent launch. A kernel launched with programmatic stream
// serialization may be scheduled while its predecessor on the stream is still
// running; pdl_wait() blocks until the predecessor has completed and its writes
// are visible (a no-op when there is no such predecessor).
// pdl_launch_dependents() lets the next kernel be scheduled from this point on.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ float key_to_float(uint32_t k) {
  uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  return __uint_as_float(u);
}

// ---------------------------------------------------------------------------
// Score problem description (host + device)
// ---------------------------------------------------------------------------
struct ScoreProblem {
  const void* q;
  int64_t q_sb, q_sh, q_ss, q_sd;
  int Lq;
  const void* k;
  const void* v;
  int64_t kv_sh;  // elements between consecutive KV heads of K and V (Lk * D if contiguous)
  int64_t kv_sb;  // elements between consecutive sequences (Hkv * kv_sh if contiguous)
  int64_t kv_ss;  // elements between consecutive keys (D if contiguous); rows of D contiguous
  int B, Hq, Hkv, Lk, D;
  int W;       // query rows per head used (window)
  int g;       // Hq / Hkv
  int M;       // g * W
  float scale; // 1 / sqrt(D)
  float eps;
  int round_mode;
  float* scores;  // [B*Hkv, Lk]
  int* status;    // where the tensor-core scorer ORs its status bits (nullptr: its own workspace word)
};

// Scratch layout of the split-K scorer (fp32 regions, 256-byte aligned).
struct ScorePlan {
  int BH;
  int tile;     // keys per split tile
  int tiles;    // ceil(Lk / tile)
  int splits;   // split-K factor
  int tps;      // tiles per split
  size_t off_pm, off_ps, off_py, off_lse, off_yn, off_y;
  size_t bytes;
};

int num_sms_current_device();
ScorePlan plan_scores(int B, int Hkv, int Lk, int M, int D);

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// A ragged batch for one call (dropkv_compress_varlen): up to kVarlenMaxSeqs
// sequences, each with its own key count and batch of (b, KV head) rows, passed to
// the selection and gather kernels by value as a kernel parameter.
constexpr int kVarlenMaxSeqs = 32;

struct VarlenSeq {
  const void* k;        // [B, Hkv, lk, D] contiguous
  const void* v;
  int64_t* keep_idx;    // [B, Hkv, cap]
  void* k_out;          // [B, Hkv, cap, D]
  void* v_out;
  int64_t score_off;    // floats before the sequence's first score row in the packed buffer
  int row0;             // its first row in the batch
  int rows;             // B * Hkv
  int lk;
  int cap;              // rows of room per (b, KV head) in keep_idx / k_out / v_out
};

struct VarlenTable {
  int n;                        // sequences
  int rows;                     // rows of the whole batch
  int protect;                  // protect window (clamped to each sequence's lk)
  int keep_window;              // window_size of the keep_len rule
  double keep_ratio;
  const int64_t* total_tokens;  // [n] on the device, or NULL (base = lk)
  const int64_t* max_keep_len;  // [n] on the device, or NULL; entries < 0 set no cap
  int32_t* keep_len_out;        // [n] on the device
  const float* scores;          // packed score rows of all sequences
  VarlenSeq s[kVarlenMaxSeqs];
};

// Sequence of batch row `row` (rows are grouped by sequence, in order).
__device__ __forceinline__ int varlen_seq_of(const VarlenTable& t, int row) {
  int s = 0;
  while (s + 1 < t.n && row >= t.s[s + 1].row0) ++s;
  return s;
}

// keep_len = min(lk, max(int(keep_ratio * base), keep_window, 1)), base =
// total_tokens or lk, then min(max_keep_len) (dropkv_cache.py:470-473; Python's
// int() of a double product truncates toward zero, as the conversion here does),
// and at most the sequence's output room.
__device__ __forceinline__ int varlen_keep_len(const VarlenTable& t, int s) {
  const int lk = t.s[s].lk;
  const double base = t.total_tokens ? (double)t.total_tokens[s] : (double)lk;
  const double prod = t.keep_ratio * base;
  long long kl = prod >= (double)lk ? (long long)lk : (long long)prod;
  kl = kl < t.keep_window ? t.keep_window : kl;
  kl = kl < 1 ? 1 : kl;
  kl = kl > lk ? lk : kl;
  if (t.max_keep_len && t.max_keep_len[s] >= 0 && t.max_keep_len[s] < kl) kl = t.max_keep_len[s];
  return (int)(kl > t.s[s].cap ? t.s[s].cap : kl);
}

// One bit per device (index < 64) recording that a per-device set-up step (kernel
// attributes) has run.  Several host threads may call into the library at once:
// the bits are read and set atomically, and a set-up step that two threads race
// on runs twice, which is harmless because each step is idempotent.
struct DeviceOnce {
  std::atomic<unsigned long long> bits{0};
  bool done(int dev) const { return dev >= 0 && dev < 64 && ((bits.load(std::memory_order_acquire) >> dev) & 1ull); }
  void mark(int dev) {
    if (dev >= 0 && dev < 64) bits.fetch_or(1ull << dev, std::memory_order_release);
  }
};

// Launchers implemented per translation unit.
int launch_scores_simt(const ScoreProblem& p, const ScorePlan& plan, void* ws, cudaStream_t st,
                       int dtype);
bool tc_supported(int dtype, int M, int D, int BH, int Lk);
size_t tc_workspace_bytes(int M, int D, int BH, int Lk);
size_t tc_status_offset(int M, int D, int BH, int Lk);
int launch_scores_tc(const ScoreProblem& p, int dtype, void* ws, cudaStream_t st);
void tc_test_set_wait_ns(uint64_t ns);
void tc_test_block_barrier(int on);

struct SelectPlan {
  size_t off_keys;   // uint32 [BH, Lk]
  size_t bytes;
};
SelectPlan plan_select(int BH, int Lk);
int launch_select(const float* scores, int BH, int Lk, int kernel_size, int protect, int keep_len,
                  int64_t* keep_idx, void* ws, cudaStream_t st);
bool select_gather_supported(int Lk, int kernel_size);

// Decode attention over the (compressed) cache (decode_attn.cu).
size_t decode_attention_workspace_size(int B, int Hq, int Hkv, int Lq, int L, int D);
// k_new != nullptr: keys [pos, L) are read from k_new / v_new ([B, Hkv, L - pos, D]
// rows with strides new_sb, new_sh) and stored into k / v at rows [pos, L).
int launch_decode_attention(const void* q, int64_t q_sb, int64_t q_sh, int64_t q_ss, int64_t q_sd, int Lq,
                            const void* k, const void* v, int64_t kv_sb, int64_t kv_sh, int dtype, int B, int Hq,
                            int Hkv, int L, int D, float scale, void* out, void* ws, cudaStream_t st,
                            const void* k_new = nullptr, const void* v_new = nullptr, int64_t new_sb = 0,
                            int64_t new_sh = 0, int pos = 0);
// k == nullptr: selection only (keep_idx), no gather
// in_sh / out_sh: elements between consecutive heads of K/V and of K_c/V_c
// (0: contiguous, Lk * D and keep_len * D)
// in_sb / in_ss (0: Hkv * in_sh and D): elements between consecutive sequences
// and keys of K/V (row bh = b * Hkv + h).
int launch_select_gather(const float* scores, int BH, int Lk, int kernel_size, int protect, int keep_len,
                         int64_t* keep_idx, const void* k, const void* v, int elem_bytes, int D, void* ko,
                         void* vo, cudaStream_t st, int64_t in_sh = 0, int64_t out_sh = 0, int Hkv = 1,
                         int64_t in_sb = 0, int64_t in_ss = 0);
int launch_gather(const void* k, const void* v, int elem_bytes, int BH, int Lk, int D,
                  const int64_t* keep_idx, int keep_len, void* k_out, void* v_out,
                  cudaStream_t st, int64_t in_sh = 0, int64_t out_sh = 0, int Hkv = 1, int64_t in_sb = 0,
                  int64_t in_ss = 0);
// A ragged batch: one selection launch and one gather launch over every row of
// the table (t.scores filled); the longest row must pass select_gather_supported.
int launch_select_gather_varlen(const VarlenTable& t, int kernel_size, int elem_bytes, int D, cudaStream_t st);

}  // namespace dropkv
