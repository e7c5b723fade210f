// extern "C" entry points of libdropkv_b200.so: argument checks, scratch
// planning and the launch sequence of each public operation.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <mutex>

#include "common.cuh"

namespace dropkv {

static thread_local std::string g_err;

void set_error(const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_err = buf;
}

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

static std::atomic<uint64_t> g_launches{0};

int check_launch(const char* what, int launches) {
  g_launches.fetch_add((uint64_t)launches, std::memory_order_relaxed);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(DROPKV_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return DROPKV_OK;
}

int num_sms_current_device() {
  static std::atomic<int> cache[64];  // zero: not queried yet
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev >= 0 && dev < 64) {
    const int c = cache[dev].load(std::memory_order_relaxed);
    if (c > 0) return c;
  }
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
  if (dev >= 0 && dev < 64) cache[dev].store(n, std::memory_order_relaxed);
  return n;
}

int simt_max_splits();
int simt_tile();

ScorePlan plan_scores(int B, int Hkv, int Lk, int M, int D) {
  ScorePlan p;
  std::memset(&p, 0, sizeof(p));
  p.BH = B * Hkv;
  p.tile = simt_tile();
  p.tiles = (Lk + p.tile - 1) / p.tile;
  const int target = 2 * num_sms_current_device();
  int s = (target + p.BH - 1) / p.BH;
  s = std::min(s, std::max(1, p.tiles / 4));
  s = std::min(s, simt_max_splits());
  s = std::max(s, 1);
  p.tps = (p.tiles + s - 1) / s;
  p.splits = (p.tiles + p.tps - 1) / p.tps;  // no empty split
  const size_t rows = (size_t)p.BH * p.splits * M;
  size_t off = 0;
  p.off_pm = off; off = align_up(off + rows * 4, 256);
  p.off_ps = off; off = align_up(off + rows * 4, 256);
  p.off_py = off; off = align_up(off + rows * D * 4, 256);
  p.off_lse = off; off = align_up(off + (size_t)p.BH * M * 4, 256);
  p.off_yn = off; off = align_up(off + (size_t)p.BH * M * 4, 256);
  p.off_y = off; off = align_up(off + (size_t)p.BH * M * D * 4, 256);
  p.bytes = off;
  return p;
}

static bool d_supported(int D) { return D == 32 || D == 64 || D == 128 || D == 256; }

static int elem_bytes_of(int dtype) {
  switch (dtype) {
    case DROPKV_DTYPE_F32: return 4;
    case DROPKV_DTYPE_F16: return 2;
    case DROPKV_DTYPE_BF16: return 2;
    default: return 0;
  }
}

static int check_score_args(const void* q, int Lq, const void* k, const void* v, int dtype, int B,
                            int Hq, int Hkv, int Lk, int D, int window, int round_p) {
  if (!q || !k || !v) return fail(DROPKV_ERR_ARG, "Q, K and V must be non-NULL device pointers");
  if (!elem_bytes_of(dtype)) return fail(DROPKV_ERR_ARG, "unknown dtype %d", dtype);
  if (B < 1 || Hq < 1 || Hkv < 1 || Lk < 1 || Lq < 1 || D < 1)
    return fail(DROPKV_ERR_ARG, "all sizes must be positive (B=%d Hq=%d Hkv=%d Lq=%d Lk=%d D=%d)", B, Hq, Hkv, Lq, Lk, D);
  if (Hq % Hkv != 0) return fail(DROPKV_ERR_ARG, "Hq (%d) must be divisible by Hkv (%d)", Hq, Hkv);
  if (window < 1) return fail(DROPKV_ERR_ARG, "window_size must be a positive int, got %d", window);
  if (Lq < window) return fail(DROPKV_ERR_ARG, "Lq (%d) must be >= window_size (%d)", Lq, window);
  if (Lk < window) return fail(DROPKV_ERR_ARG, "Lk (%d) must be >= window_size (%d)", Lk, window);
  if (Lq > Lk) return fail(DROPKV_ERR_ARG, "Lq (%d) must be <= Lk (%d) (Q must be tail-aligned suffix)", Lq, Lk);
  if ((int64_t)B * Hkv > 65535) return fail(DROPKV_ERR_ARG, "B*Hkv (%lld) exceeds 65535", (long long)B * Hkv);
  if (!d_supported(D)) return fail(DROPKV_ERR_UNSUPPORTED, "head_dim %d not supported (32, 64, 128, 256)", D);
  if (round_p < DROPKV_ROUND_NONE || round_p > DROPKV_ROUND_F16) return fail(DROPKV_ERR_ARG, "bad round_p %d", round_p);
  if ((reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v)) % 16)
    return fail(DROPKV_ERR_ARG, "K and V must be 16-byte aligned");
  return DROPKV_OK;
}

static ScoreProblem make_problem(const void* q, int64_t q_sb, int64_t q_sh, int64_t q_ss, int64_t q_sd,
                                 int Lq, const void* k, const void* v, int B, int Hq, int Hkv, int Lk,
                                 int D, int window, float eps, int round_p, float* scores) {
  ScoreProblem p;
  p.q = q; p.q_sb = q_sb; p.q_sh = q_sh; p.q_ss = q_ss; p.q_sd = q_sd; p.Lq = Lq;
  p.k = k; p.v = v; p.kv_sh = (int64_t)Lk * D; p.kv_sb = (int64_t)Hkv * Lk * D; p.kv_ss = D; p.B = B; p.Hq = Hq; p.Hkv = Hkv; p.Lk = Lk; p.D = D;
  p.W = window; p.g = Hq / Hkv; p.M = p.g * window;
  p.scale = (float)(1.0 / std::sqrt((double)D));
  p.eps = eps; p.round_mode = round_p; p.scores = scores; p.status = nullptr;
  return p;
}

static int check_ws(void* ws, size_t have, size_t need) {
  if (need == 0) return DROPKV_OK;
  if (!ws) return fail(DROPKV_ERR_WORKSPACE, "workspace is NULL (%zu bytes needed)", need);
  if (have < need) return fail(DROPKV_ERR_WORKSPACE, "workspace too small: %zu < %zu bytes", have, need);
  if (reinterpret_cast<uintptr_t>(ws) % 256) return fail(DROPKV_ERR_WORKSPACE, "workspace must be 256-byte aligned");
  return DROPKV_OK;
}

static std::atomic<int> g_backend{0};  // 0 auto, 1 CUDA-core scorer, 2 tensor-core scorer

static bool use_tc(int dtype, int B, int Hkv, int Lk, int M, int D) {
  const int be = g_backend.load(std::memory_order_relaxed);
  if (be == 1) return false;
  return tc_supported(dtype, M, D, B * Hkv, Lk);
}

static size_t scores_ws_bytes(int dtype, int B, int Hkv, int Lk, int M, int D) {
  if (use_tc(dtype, B, Hkv, Lk, M, D)) return tc_workspace_bytes(M, D, B * Hkv, Lk);
  return plan_scores(B, Hkv, Lk, M, D).bytes;
}

static int run_scores(const ScoreProblem& p, int dtype, void* ws, cudaStream_t st) {
  if (use_tc(dtype, p.B, p.Hkv, p.Lk, p.M, p.D)) return launch_scores_tc(p, dtype, ws, st);
  if (g_backend.load(std::memory_order_relaxed) == 2)
    return fail(DROPKV_ERR_UNSUPPORTED, "tensor-core scorer forced but it does not cover this problem");
  if (p.kv_ss != p.D || p.kv_sb != (int64_t)p.Hkv * p.kv_sh)
    return fail(DROPKV_ERR_UNSUPPORTED, "the CUDA-core scorer (fp32, D 32/256, M > 64) needs K/V rows packed "
                                        "per (sequence, head); copy K and V to that layout first");
  ScorePlan plan = plan_scores(p.B, p.Hkv, p.Lk, p.M, p.D);
  return launch_scores_simt(p, plan, ws, st, dtype);
}

static int check_select_args(int B, int Hkv, int Lk, int kernel_size, int protect, int keep_len) {
  if (B < 1 || Hkv < 1 || Lk < 1) return fail(DROPKV_ERR_ARG, "B, Hkv and Lk must be positive");
  if ((int64_t)B * Hkv > 2147483647) return fail(DROPKV_ERR_ARG, "B*Hkv too large");
  if (kernel_size < 1 || kernel_size % 2 == 0)
    return fail(DROPKV_ERR_ARG, "kernel_size must be a positive odd integer, got %d", kernel_size);
  if (protect < 0) return fail(DROPKV_ERR_ARG, "protect window must be >= 0, got %d", protect);
  if (keep_len < 1 || keep_len > Lk)
    return fail(DROPKV_ERR_ARG, "keep_len must be in [1, Lk=%d], got %d", Lk, keep_len);
  return DROPKV_OK;
}

// Scratch of dropkv_scores_static: a device array of this module, so the call
// needs no allocation.  Its address is looked up once per device (with that device
// current) and cached.
static __device__ __align__(256) unsigned char g_static_scratch[DROPKV_STATIC_SCRATCH_BYTES];
// A zero status word: what dropkv_scores_static_status copies for problems the
// CUDA-core scorer serves (it has no bounded waits, so no status of its own).
static __device__ __align__(16) int g_zero_status = 0;
static std::mutex g_static_mu;
static void* g_static_addr[64] = {nullptr};
static void* g_zero_addr[64] = {nullptr};

static int static_scratch_address(void** out, void** zero_word = nullptr) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(DROPKV_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return fail(DROPKV_ERR_UNSUPPORTED, "device index %d is beyond 63", dev);
  std::lock_guard<std::mutex> lock(g_static_mu);
  if (!g_static_addr[dev]) {
    void* p = nullptr;
    void* z = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess || !p)
      return fail(DROPKV_ERR_CUDA, "cudaGetSymbolAddress of the static scratch on device %d: %s", dev,
                  cudaGetErrorString(e));
    e = cudaGetSymbolAddress(&z, g_zero_status);
    if (e != cudaSuccess || !z)
      return fail(DROPKV_ERR_CUDA, "cudaGetSymbolAddress of the zero status word on device %d: %s", dev,
                  cudaGetErrorString(e));
    g_zero_addr[dev] = z;
    g_static_addr[dev] = p;
  }
  *out = g_static_addr[dev];
  if (zero_word) *zero_word = g_zero_addr[dev];
  return DROPKV_OK;
}

}  // namespace dropkv

using namespace dropkv;

extern "C" {

const char* dropkv_version(void) { return "dropkv_b200 0.1.0 (sm_100a)"; }

const char* dropkv_last_error(void) { return g_err.c_str(); }

uint64_t dropkv_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

size_t dropkv_scores_workspace_size(int B, int Hq, int Hkv, int Lk, int D, int window) {
  if (B < 1 || Hq < 1 || Hkv < 1 || Lk < 1 || D < 1 || window < 1 || Hq % Hkv) return 0;
  const int M = (Hq / Hkv) * window;
  size_t a = scores_ws_bytes(DROPKV_DTYPE_BF16, B, Hkv, Lk, M, D);
  size_t b = scores_ws_bytes(DROPKV_DTYPE_F32, B, Hkv, Lk, M, D);
  return a > b ? a : b;
}

size_t dropkv_scores_status_offset(int dtype, int B, int Hq, int Hkv, int Lk, int D, int window) {
  if (B < 1 || Hq < 1 || Hkv < 1 || Lk < 1 || D < 1 || window < 1 || Hq % Hkv) return (size_t)-1;
  const int M = (Hq / Hkv) * window;
  if (!use_tc(dtype, B, Hkv, Lk, M, D)) return (size_t)-1;
  return tc_status_offset(M, D, B * Hkv, Lk);
}

int dropkv_test_scorer_waits(uint64_t wait_limit_ns, int block_group_barrier) {
  tc_test_set_wait_ns(wait_limit_ns);
  tc_test_block_barrier(block_group_barrier);
  return DROPKV_OK;
}

int dropkv_set_scorer(int mode) {
  if (mode < 0 || mode > 2) return fail(DROPKV_ERR_ARG, "scorer mode must be 0 (auto), 1 (CUDA cores) or 2 (tensor cores)");
  g_backend.store(mode);
  return DROPKV_OK;
}

int dropkv_scorer_for(int dtype, int B, int Hq, int Hkv, int Lk, int D, int window) {
  if (B < 1 || Hq < 1 || Hkv < 1 || Lk < 1 || D < 1 || window < 1 || Hq % Hkv) return 0;
  return use_tc(dtype, B, Hkv, Lk, (Hq / Hkv) * window, D) ? 2 : 1;
}

int dropkv_scores(const void* q, int64_t q_sb, int64_t q_sh, int64_t q_ss, int64_t q_sd, int Lq,
                  const void* k, const void* v, int dtype, int B, int Hq, int Hkv, int Lk, int D,
                  int window, float eps, int round_p, float* scores, void* workspace,
                  size_t workspace_bytes, void* stream) {
  int rc = check_score_args(q, Lq, k, v, dtype, B, Hq, Hkv, Lk, D, window, round_p);
  if (rc) return rc;
  if (!scores) return fail(DROPKV_ERR_ARG, "scores must be a non-NULL device pointer");
  size_t need = dropkv_scores_workspace_size(B, Hq, Hkv, Lk, D, window);
  if ((rc = check_ws(workspace, workspace_bytes, need))) return rc;
  ScoreProblem p = make_problem(q, q_sb, q_sh, q_ss, q_sd, Lq, k, v, B, Hq, Hkv, Lk, D, window, eps,
                                round_p, scores);
  return run_scores(p, dtype, workspace, reinterpret_cast<cudaStream_t>(stream));
}

int dropkv_scores_static(const void* q, int64_t q_sb, int64_t q_sh, int64_t q_ss, int64_t q_sd, int Lq,
                         const void* k, const void* v, int dtype, int B, int Hq, int Hkv, int Lk, int D,
                         int window, float eps, int round_p, float* scores, void* stream) {
  int rc = check_score_args(q, Lq, k, v, dtype, B, Hq, Hkv, Lk, D, window, round_p);
  if (rc) return rc;
  if (!scores) return fail(DROPKV_ERR_ARG, "scores must be a non-NULL device pointer");
  const size_t need = scores_ws_bytes(dtype, B, Hkv, Lk, (Hq / Hkv) * window, D);
  if (need > (size_t)DROPKV_STATIC_SCRATCH_BYTES)
    return fail(DROPKV_ERR_WORKSPACE,
                "dropkv_scores_static: this problem needs %zu bytes of scratch, more than the %zu-byte "
                "static buffer; call dropkv_scores with a workspace instead",
                need, (size_t)DROPKV_STATIC_SCRATCH_BYTES);
  void* ws = nullptr;
  if ((rc = static_scratch_address(&ws))) return rc;
  ScoreProblem p = make_problem(q, q_sb, q_sh, q_ss, q_sd, Lq, k, v, B, Hq, Hkv, Lk, D, window, eps,
                                round_p, scores);
  return run_scores(p, dtype, ws, reinterpret_cast<cudaStream_t>(stream));
}

int dropkv_scores_static_status(int dtype, int B, int Hq, int Hkv, int Lk, int D, int window, int* status_out,
                                void* stream) {
  if (!status_out) return fail(DROPKV_ERR_ARG, "status_out must be non-NULL");
  if (!elem_bytes_of(dtype)) return fail(DROPKV_ERR_ARG, "unknown dtype %d", dtype);
  if (B < 1 || Hq < 1 || Hkv < 1 || Lk < 1 || D < 1 || window < 1 || Hq % Hkv)
    return fail(DROPKV_ERR_ARG, "invalid problem sizes");
  void* base = nullptr;
  void* zero = nullptr;
  int rc = static_scratch_address(&base, &zero);
  if (rc) return rc;
  const int M = (Hq / Hkv) * window;
  const void* src = use_tc(dtype, B, Hkv, Lk, M, D)
                        ? static_cast<const void*>(reinterpret_cast<char*>(base) + tc_status_offset(M, D, B * Hkv, Lk))
                        : static_cast<const void*>(zero);
  cudaError_t e = cudaMemcpyAsync(status_out, src, sizeof(int), cudaMemcpyDefault,
                                  reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(DROPKV_ERR_CUDA, "copy of the static status word: %s", cudaGetErrorString(e));
  return DROPKV_OK;
}

size_t dropkv_select_workspace_size(int B, int Hkv, int Lk) {
  if (B < 1 || Hkv < 1 || Lk < 1) return 0;
  return plan_select(B * Hkv, Lk).bytes;
}

int dropkv_select(const float* scores, int B, int Hkv, int Lk, int kernel_size, int protect_window,
                  int keep_len, int64_t* keep_idx, void* workspace, size_t workspace_bytes,
                  void* stream) {
  int rc = check_select_args(B, Hkv, Lk, kernel_size, protect_window, keep_len);
  if (rc) return rc;
  if (!scores || !keep_idx) return fail(DROPKV_ERR_ARG, "scores and keep_idx must be non-NULL");
  if ((rc = check_ws(workspace, workspace_bytes, dropkv_select_workspace_size(B, Hkv, Lk)))) return rc;
  int protect = std::min(protect_window, Lk);
  if (select_gather_supported(Lk, kernel_size))
    return launch_select_gather(scores, B * Hkv, Lk, kernel_size, protect, keep_len, keep_idx, nullptr, nullptr,
                                4, 1, nullptr, nullptr, reinterpret_cast<cudaStream_t>(stream));
  return launch_select(scores, B * Hkv, Lk, kernel_size, protect, keep_len, keep_idx, workspace,
                       reinterpret_cast<cudaStream_t>(stream));
}

int dropkv_gather(const void* k, const void* v, int elem_bytes, int B, int Hkv, int Lk, int D,
                  const int64_t* keep_idx, int keep_len, void* k_out, void* v_out, void* stream) {
  if (!k || !v || !keep_idx || !k_out || !v_out) return fail(DROPKV_ERR_ARG, "NULL pointer argument");
  if (elem_bytes != 2 && elem_bytes != 4) return fail(DROPKV_ERR_ARG, "elem_bytes must be 2 or 4");
  if (B < 1 || Hkv < 1 || Lk < 1 || D < 1 || keep_len < 0)
    return fail(DROPKV_ERR_ARG, "invalid gather sizes");
  if ((int64_t)B * Hkv > 65535) return fail(DROPKV_ERR_ARG, "B*Hkv exceeds 65535");
  return launch_gather(k, v, elem_bytes, B * Hkv, Lk, D, keep_idx, keep_len, k_out, v_out,
                       reinterpret_cast<cudaStream_t>(stream));
}

size_t dropkv_compress_workspace_size(int B, int Hq, int Hkv, int Lk, int D, int window) {
  size_t s = dropkv_scores_workspace_size(B, Hq, Hkv, Lk, D, window);
  if (!s) return 0;
  size_t sc = align_up((size_t)B * Hkv * Lk * 4, 256);
  return s + sc + dropkv_select_workspace_size(B, Hkv, Lk);
}

int dropkv_compress(const void* q, int64_t q_sb, int64_t q_sh, int64_t q_ss, int64_t q_sd, int Lq,
                    const void* k, const void* v, int dtype, int B, int Hq, int Hkv, int Lk, int D,
                    int window, float eps, int round_p, int kernel_size, int protect_window,
                    int keep_len, float* scores_out, int64_t* keep_idx, void* k_out, void* v_out,
                    void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_score_args(q, Lq, k, v, dtype, B, Hq, Hkv, Lk, D, window, round_p);
  if (rc) return rc;
  if ((rc = check_select_args(B, Hkv, Lk, kernel_size, protect_window, keep_len))) return rc;
  if (!keep_idx || !k_out || !v_out) return fail(DROPKV_ERR_ARG, "keep_idx, k_out and v_out must be non-NULL");
  size_t s_ws = dropkv_scores_workspace_size(B, Hq, Hkv, Lk, D, window);
  size_t need = dropkv_compress_workspace_size(B, Hq, Hkv, Lk, D, window);
  if ((rc = check_ws(workspace, workspace_bytes, need))) return rc;
  char* base = reinterpret_cast<char*>(workspace);
  float* scores = scores_out ? scores_out : reinterpret_cast<float*>(base + s_ws);
  void* sel_ws = base + s_ws + align_up((size_t)B * Hkv * Lk * 4, 256);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  ScoreProblem p = make_problem(q, q_sb, q_sh, q_ss, q_sd, Lq, k, v, B, Hq, Hkv, Lk, D, window, eps,
                                round_p, scores);
  if ((rc = run_scores(p, dtype, workspace, st))) return rc;
  int protect = std::min(protect_window, Lk);
  if (select_gather_supported(Lk, kernel_size))
    return launch_select_gather(scores, B * Hkv, Lk, kernel_size, protect, keep_len, keep_idx, k, v,
                                elem_bytes_of(dtype), D, k_out, v_out, st);
  if ((rc = launch_select(scores, B * Hkv, Lk, kernel_size, protect, keep_len, keep_idx, sel_ws, st))) return rc;
  return launch_gather(k, v, elem_bytes_of(dtype), B * Hkv, Lk, D, keep_idx, keep_len, k_out, v_out, st);
}

int dropkv_compress_strided(const void* q, int64_t q_sb, int64_t q_sh, int64_t q_ss, int64_t q_sd, int Lq,
                            const void* k, const void* v, int64_t kv_head_stride, int dtype, int B, int Hq,
                            int Hkv, int Lk, int D, int window, float eps, int round_p, int kernel_size,
                            int protect_window, int keep_len, float* scores_out, int64_t* keep_idx,
                            void* k_out, void* v_out, int64_t out_head_stride, void* workspace,
                            size_t workspace_bytes, void* stream) {
  int rc = check_score_args(q, Lq, k, v, dtype, B, Hq, Hkv, Lk, D, window, round_p);
  if (rc) return rc;
  if ((rc = check_select_args(B, Hkv, Lk, kernel_size, protect_window, keep_len))) return rc;
  if (!keep_idx || !k_out || !v_out) return fail(DROPKV_ERR_ARG, "keep_idx, k_out and v_out must be non-NULL");
  if (kv_head_stride < (int64_t)Lk * D || kv_head_stride % 8)
    return fail(DROPKV_ERR_ARG, "kv_head_stride (%lld) must be >= Lk*D (%lld) and a multiple of 8",
                (long long)kv_head_stride, (long long)Lk * D);
  if (out_head_stride < (int64_t)keep_len * D || out_head_stride % 8)
    return fail(DROPKV_ERR_ARG, "out_head_stride (%lld) must be >= keep_len*D (%lld) and a multiple of 8",
                (long long)out_head_stride, (long long)keep_len * D);
  if (reinterpret_cast<uintptr_t>(k_out) % 16 || reinterpret_cast<uintptr_t>(v_out) % 16)
    return fail(DROPKV_ERR_ARG, "k_out and v_out must be 16-byte aligned");
  size_t s_ws = dropkv_scores_workspace_size(B, Hq, Hkv, Lk, D, window);
  size_t need = dropkv_compress_workspace_size(B, Hq, Hkv, Lk, D, window);
  if ((rc = check_ws(workspace, workspace_bytes, need))) return rc;
  char* base = reinterpret_cast<char*>(workspace);
  float* scores = scores_out ? scores_out : reinterpret_cast<float*>(base + s_ws);
  void* sel_ws = base + s_ws + align_up((size_t)B * Hkv * Lk * 4, 256);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  ScoreProblem p = make_problem(q, q_sb, q_sh, q_ss, q_sd, Lq, k, v, B, Hq, Hkv, Lk, D, window, eps,
                                round_p, scores);
  p.kv_sh = kv_head_stride;
  p.kv_sb = (int64_t)Hkv * kv_head_stride;
  if ((rc = run_scores(p, dtype, workspace, st))) return rc;
  int protect = std::min(protect_window, Lk);
  if (select_gather_supported(Lk, kernel_size))
    return launch_select_gather(scores, B * Hkv, Lk, kernel_size, protect, keep_len, keep_idx, k, v,
                                elem_bytes_of(dtype), D, k_out, v_out, st, kv_head_stride, out_head_stride);
  if ((rc = launch_select(scores, B * Hkv, Lk, kernel_size, protect, keep_len, keep_idx, sel_ws, st))) return rc;
  return launch_gather(k, v, elem_bytes_of(dtype), B * Hkv, Lk, D, keep_idx, keep_len, k_out, v_out, st,
                       kv_head_stride, out_head_stride);
}

int dropkv_compress_kv_strides(const void* q, int64_t q_sb, int64_t q_sh, int64_t q_ss, int64_t q_sd, int Lq,
                               const void* k, const void* v, int64_t kv_sb, int64_t kv_sh, int64_t kv_ss,
                               int dtype, int B, int Hq, int Hkv, int Lk, int D, int window, float eps, int round_p,
                               int kernel_size, int protect_window, int keep_len, float* scores_out,
                               int64_t* keep_idx, void* k_out, void* v_out, void* workspace,
                               size_t workspace_bytes, void* stream) {
  int rc = check_score_args(q, Lq, k, v, dtype, B, Hq, Hkv, Lk, D, window, round_p);
  if (rc) return rc;
  if ((rc = check_select_args(B, Hkv, Lk, kernel_size, protect_window, keep_len))) return rc;
  if (!keep_idx || !k_out || !v_out) return fail(DROPKV_ERR_ARG, "keep_idx, k_out and v_out must be non-NULL");
  const int eb = elem_bytes_of(dtype);
  if (kv_ss < D || kv_sh < 1 || kv_sb < 1 || (kv_ss * eb) % 16 || (kv_sh * eb) % 16 || (kv_sb * eb) % 16)
    return fail(DROPKV_ERR_ARG, "K/V strides (%lld, %lld, %lld) must be positive multiples of 16 bytes with rows "
                "of D=%d contiguous elements", (long long)kv_sb, (long long)kv_sh, (long long)kv_ss, D);
  size_t s_ws = dropkv_scores_workspace_size(B, Hq, Hkv, Lk, D, window);
  size_t need = dropkv_compress_workspace_size(B, Hq, Hkv, Lk, D, window);
  if ((rc = check_ws(workspace, workspace_bytes, need))) return rc;
  char* base = reinterpret_cast<char*>(workspace);
  float* scores = scores_out ? scores_out : reinterpret_cast<float*>(base + s_ws);
  void* sel_ws = base + s_ws + align_up((size_t)B * Hkv * Lk * 4, 256);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  ScoreProblem p = make_problem(q, q_sb, q_sh, q_ss, q_sd, Lq, k, v, B, Hq, Hkv, Lk, D, window, eps,
                                round_p, scores);
  p.kv_sb = kv_sb;
  p.kv_sh = kv_sh;
  p.kv_ss = kv_ss;
  if ((rc = run_scores(p, dtype, workspace, st))) return rc;
  int protect = std::min(protect_window, Lk);
  if (select_gather_supported(Lk, kernel_size))
    return launch_select_gather(scores, B * Hkv, Lk, kernel_size, protect, keep_len, keep_idx, k, v, eb, D, k_out,
                                v_out, st, kv_sh, 0, Hkv, kv_sb, kv_ss);
  if ((rc = launch_select(scores, B * Hkv, Lk, kernel_size, protect, keep_len, keep_idx, sel_ws, st))) return rc;
  return launch_gather(k, v, eb, B * Hkv, Lk, D, keep_idx, keep_len, k_out, v_out, st, kv_sh, 0, Hkv, kv_sb, kv_ss);
}


int dropkv_append_rows(void* k_dst, void* v_dst, int64_t dst_head_stride, int dst_row, const void* k_src,
                       const void* v_src, int64_t src_head_stride, int rows, int D, int elem_bytes, int BH,
                       void* stream) {
  if (!k_dst || !v_dst || !k_src || !v_src) return fail(DROPKV_ERR_ARG, "NULL pointer argument");
  if (elem_bytes != 2 && elem_bytes != 4) return fail(DROPKV_ERR_ARG, "elem_bytes must be 2 or 4");
  if (rows < 0 || D < 1 || BH < 1 || dst_row < 0) return fail(DROPKV_ERR_ARG, "invalid append sizes");
  if (src_head_stride < (int64_t)rows * D || dst_head_stride < (int64_t)(dst_row + rows) * D)
    return fail(DROPKV_ERR_ARG, "head strides too small for the rows");
  if (rows == 0) return DROPKV_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const size_t width = (size_t)rows * D * elem_bytes;
  const size_t off = (size_t)dst_row * D * elem_bytes;
  for (int t = 0; t < 2; ++t) {
    char* dst = reinterpret_cast<char*>(t ? v_dst : k_dst) + off;
    const void* src = t ? v_src : k_src;
    cudaError_t e = cudaMemcpy2DAsync(dst, (size_t)dst_head_stride * elem_bytes, src,
                                      (size_t)src_head_stride * elem_bytes, width, (size_t)BH,
                                      cudaMemcpyDeviceToDevice, st);
    if (e != cudaSuccess) return fail(DROPKV_ERR_CUDA, "append copy: %s", cudaGetErrorString(e));
  }
  return DROPKV_OK;
}

size_t dropkv_decode_attention_workspace_size(int B, int Hq, int Hkv, int Lq, int L, int D) {
  if (B < 1 || Hq < 1 || Hkv < 1 || Hq % Hkv || Lq < 1 || L < Lq || (D != 64 && D != 128)) return 0;
  return decode_attention_workspace_size(B, Hq, Hkv, Lq, L, D);
}

int dropkv_decode_attention(const void* q, int64_t q_sb, int64_t q_sh, int64_t q_ss, int64_t q_sd, int Lq,
                            const void* k, const void* v, int64_t kv_sb, int64_t kv_sh, int dtype, int B, int Hq,
                            int Hkv, int L, int D, float scale, void* out, void* workspace, size_t workspace_bytes,
                            void* stream) {
  if (!q || !k || !v || !out) return fail(DROPKV_ERR_ARG, "NULL pointer argument");
  if (dtype != DROPKV_DTYPE_BF16 && dtype != DROPKV_DTYPE_F16)
    return fail(DROPKV_ERR_UNSUPPORTED, "decode attention takes bf16 or fp16 inputs");
  if (D != 64 && D != 128) return fail(DROPKV_ERR_UNSUPPORTED, "decode attention needs D of 64 or 128 (got %d)", D);
  if (B < 1 || Hq < 1 || Hkv < 1 || Hq % Hkv) return fail(DROPKV_ERR_ARG, "invalid head counts Hq=%d Hkv=%d", Hq, Hkv);
  if (Lq < 1 || L < Lq) return fail(DROPKV_ERR_ARG, "need 1 <= Lq <= L (Lq=%d, L=%d)", Lq, L);
  if ((int64_t)B * Hkv > 65535) return fail(DROPKV_ERR_ARG, "B*Hkv exceeds 65535");
  if (kv_sh < (int64_t)L * D || kv_sb < (int64_t)Hkv * kv_sh) return fail(DROPKV_ERR_ARG, "K/V strides too small");
  if ((reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v)) % 16 || (kv_sh * 2) % 16 || (kv_sb * 2) % 16)
    return fail(DROPKV_ERR_ARG, "K/V rows must start on 16-byte boundaries");
  if (!(scale > 0.f)) return fail(DROPKV_ERR_ARG, "scale must be positive");
  int rc = check_ws(workspace, workspace_bytes, dropkv_decode_attention_workspace_size(B, Hq, Hkv, Lq, L, D));
  if (rc) return rc;
  return launch_decode_attention(q, q_sb, q_sh, q_ss, q_sd, Lq, k, v, kv_sb, kv_sh, dtype, B, Hq, Hkv, L, D, scale,
                                 out, workspace, reinterpret_cast<cudaStream_t>(stream));
}

// ---------------------------------------------------------------------------
// Ragged batch: one call, keep_len per sequence on the device
// ---------------------------------------------------------------------------
// Workspace: [256 B: OR of the scorers' status words][scorer scratch, the largest
// any sequence needs (the scorer launches run one after another on the stream)]
// [each sequence's score rows, 256-byte aligned].
static size_t varlen_layout(int n_seq, const dropkv_varlen_seq* seqs, int Hq, int Hkv, int D, int window,
                            size_t* off_scores, int64_t* score_off /* [n_seq] floats, may be NULL */) {
  size_t scratch = 0;
  for (int i = 0; i < n_seq; ++i) {
    const int W = std::min(window, seqs[i].Lq);
    scratch = std::max(scratch, dropkv_scores_workspace_size(seqs[i].B, Hq, Hkv, seqs[i].Lk, D, W));
  }
  const size_t off = align_up(256 + scratch, 256);
  size_t bytes = off;
  for (int i = 0; i < n_seq; ++i) {
    if (score_off) score_off[i] = (int64_t)((bytes - off) / 4);
    bytes = align_up(bytes + (size_t)seqs[i].B * Hkv * seqs[i].Lk * 4, 256);
  }
  if (off_scores) *off_scores = off;
  return bytes;
}

size_t dropkv_compress_varlen_workspace_size(int n_seq, const dropkv_varlen_seq* seqs, int Hq, int Hkv, int D,
                                             int window) {
  if (n_seq < 1 || n_seq > DROPKV_VARLEN_MAX_SEQS || !seqs || Hq < 1 || Hkv < 1 || D < 1 || window < 1) return 0;
  for (int i = 0; i < n_seq; ++i)
    if (seqs[i].B < 1 || seqs[i].Lk < 1 || seqs[i].Lq < 1) return 0;
  return varlen_layout(n_seq, seqs, Hq, Hkv, D, window, nullptr, nullptr);
}

int dropkv_compress_varlen(int n_seq, const dropkv_varlen_seq* seqs, int dtype, int Hq, int Hkv, int D, int window,
                           float eps, int round_p, int kernel_size, int protect_window, double keep_ratio,
                           int keep_window, const int64_t* total_tokens, const int64_t* max_keep_len,
                           int32_t* keep_len_out, void* workspace, size_t workspace_bytes, void* stream) {
  if (n_seq < 1 || n_seq > DROPKV_VARLEN_MAX_SEQS)
    return fail(DROPKV_ERR_ARG, "n_seq must be in [1, %d], got %d", DROPKV_VARLEN_MAX_SEQS, n_seq);
  if (!seqs || !keep_len_out) return fail(DROPKV_ERR_ARG, "seqs and keep_len_out must be non-NULL");
  if (!(keep_ratio > 0.0 && keep_ratio <= 1.0))
    return fail(DROPKV_ERR_ARG, "keep_ratio must be in (0, 1], got %g", keep_ratio);
  if (keep_window < 0) return fail(DROPKV_ERR_ARG, "keep_window must be >= 0, got %d", keep_window);
  if (window < 1) return fail(DROPKV_ERR_ARG, "window_size must be a positive int, got %d", window);
  int64_t rows = 0;
  for (int i = 0; i < n_seq; ++i) {
    const dropkv_varlen_seq& q = seqs[i];
    const int W = std::min(window, q.Lq);
    int rc = check_score_args(q.q, q.Lq, q.k, q.v, dtype, q.B, Hq, Hkv, q.Lk, D, W, round_p);
    if (!rc) rc = check_select_args(q.B, Hkv, q.Lk, kernel_size, protect_window, 1);
    if (rc) return fail(rc, "sequence %d: %s", i, dropkv_last_error());
    if (q.cap < 1 || q.cap > q.Lk) return fail(DROPKV_ERR_ARG, "sequence %d: cap must be in [1, Lk=%d], got %d", i, q.Lk, q.cap);
    if (!q.keep_idx || !q.k_out || !q.v_out)
      return fail(DROPKV_ERR_ARG, "sequence %d: keep_idx, k_out and v_out must be non-NULL", i);
    if (!select_gather_supported(q.Lk, kernel_size))
      return fail(DROPKV_ERR_UNSUPPORTED, "sequence %d: %d keys exceed the one-launch selection", i, q.Lk);
    rows += (int64_t)q.B * Hkv;
  }
  if (rows > 65535) return fail(DROPKV_ERR_ARG, "the batch has %lld (b, KV head) rows; at most 65535", (long long)rows);
  VarlenTable t;
  std::memset(&t, 0, sizeof(t));
  size_t off_scores;
  int64_t score_off[DROPKV_VARLEN_MAX_SEQS];
  const size_t need = varlen_layout(n_seq, seqs, Hq, Hkv, D, window, &off_scores, score_off);
  int rc = check_ws(workspace, workspace_bytes, need);
  if (rc) return rc;
  char* base = reinterpret_cast<char*>(workspace);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int* status = reinterpret_cast<int*>(base);
  cudaError_t e = cudaMemsetAsync(status, 0, 4, st);
  if (e != cudaSuccess) return fail(DROPKV_ERR_CUDA, "status reset: %s", cudaGetErrorString(e));
  t.n = n_seq;
  t.protect = protect_window;
  t.keep_window = keep_window;
  t.keep_ratio = keep_ratio;
  t.total_tokens = total_tokens;
  t.max_keep_len = max_keep_len;
  t.keep_len_out = keep_len_out;
  t.scores = reinterpret_cast<const float*>(base + off_scores);
  int row0 = 0;
  for (int i = 0; i < n_seq; ++i) {
    const dropkv_varlen_seq& q = seqs[i];
    float* sc = reinterpret_cast<float*>(base + off_scores) + score_off[i];
    ScoreProblem p = make_problem(q.q, q.q_sb, q.q_sh, q.q_ss, q.q_sd, q.Lq, q.k, q.v, q.B, Hq, Hkv, q.Lk, D,
                                  std::min(window, q.Lq), eps, round_p, sc);
    p.status = status;
    if ((rc = run_scores(p, dtype, base + 256, st))) return rc;
    VarlenSeq& v = t.s[i];
    v.k = q.k;
    v.v = q.v;
    v.keep_idx = q.keep_idx;
    v.k_out = q.k_out;
    v.v_out = q.v_out;
    v.score_off = score_off[i];
    v.row0 = row0;
    v.rows = q.B * Hkv;
    v.lk = q.Lk;
    v.cap = q.cap;
    row0 += v.rows;
  }
  t.rows = row0;
  return launch_select_gather_varlen(t, kernel_size, elem_bytes_of(dtype), D, st);
}

int dropkv_decode_append_attention(const void* q, int64_t q_sb, int64_t q_sh, int64_t q_ss, int64_t q_sd, int Lq,
                                   const void* k_new, const void* v_new, int64_t new_sb, int64_t new_sh, int n_new,
                                   void* k, void* v, int64_t kv_sb, int64_t kv_sh, int pos, int dtype, int B,
                                   int Hq, int Hkv, int D, float scale, void* out, void* workspace,
                                   size_t workspace_bytes, void* stream) {
  if (!q || !k || !v || !out || !k_new || !v_new) return fail(DROPKV_ERR_ARG, "NULL pointer argument");
  if (dtype != DROPKV_DTYPE_BF16 && dtype != DROPKV_DTYPE_F16)
    return fail(DROPKV_ERR_UNSUPPORTED, "decode attention takes bf16 or fp16 inputs");
  if (D != 64 && D != 128) return fail(DROPKV_ERR_UNSUPPORTED, "decode attention needs D of 64 or 128 (got %d)", D);
  if (B < 1 || Hq < 1 || Hkv < 1 || Hq % Hkv) return fail(DROPKV_ERR_ARG, "invalid head counts Hq=%d Hkv=%d", Hq, Hkv);
  if (n_new < 1 || pos < 0) return fail(DROPKV_ERR_ARG, "need n_new >= 1 and pos >= 0 (n_new=%d, pos=%d)", n_new, pos);
  const int L = pos + n_new;
  if (Lq < 1 || L < Lq) return fail(DROPKV_ERR_ARG, "need 1 <= Lq <= pos + n_new (Lq=%d, L=%d)", Lq, L);
  if ((int64_t)B * Hkv > 65535) return fail(DROPKV_ERR_ARG, "B*Hkv exceeds 65535");
  if (kv_sh < (int64_t)L * D || kv_sb < (int64_t)Hkv * kv_sh)
    return fail(DROPKV_ERR_ARG, "K/V buffer strides too small for %d rows", L);
  if (new_sh < (int64_t)n_new * D || new_sb < (int64_t)Hkv * new_sh)
    return fail(DROPKV_ERR_ARG, "new-row strides too small for %d rows", n_new);
  if ((reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(k_new) |
       reinterpret_cast<uintptr_t>(v_new)) % 16 ||
      (kv_sh * 2) % 16 || (kv_sb * 2) % 16 || (new_sh * 2) % 16 || (new_sb * 2) % 16)
    return fail(DROPKV_ERR_ARG, "K/V rows must start on 16-byte boundaries");
  if (!(scale > 0.f)) return fail(DROPKV_ERR_ARG, "scale must be positive");
  int rc = check_ws(workspace, workspace_bytes, dropkv_decode_attention_workspace_size(B, Hq, Hkv, Lq, L, D));
  if (rc) return rc;
  return launch_decode_attention(q, q_sb, q_sh, q_ss, q_sd, Lq, k, v, kv_sb, kv_sh, dtype, B, Hq, Hkv, L, D, scale,
                                 out, workspace, reinterpret_cast<cudaStream_t>(stream), k_new, v_new, new_sb, new_sh,
                                 pos);
}

}  // extern "C"

