// Split-K DropKV scoring on CUDA cores (fp32 arithmetic for every input dtype).
//
// This is the general scorer: any dtype (fp32 / fp16 / bf16), D in {32, 64, 128,
// 256}, any window and GQA group size.  The tensor-core scorer in scores_tc.cu
// takes bf16/fp16 inputs with D in {64, 128}; this one covers everything else and
// is the fp32-exact path (scores within 1e-5 of the reference for fp32 inputs).
//
// Three launches per call, all on the caller's stream:
//   1. fwd_partial: grid (splits, B*Hkv).  Each CTA streams a contiguous key range
//      of one head and keeps an online softmax over the head's M = g*W window rows:
//      running max m, running sum s and unnormalised y = sum_j exp(l_mj - m) v_j.
//      (reference: dropkv_triton.py:290-387, split-K forward)
//   2. merge: grid (B*Hkv).  Merges the split partials with the max-rescale rule
//      into lse_m, y_m = softmax(l_m) V and ||y_m||^2 (dropkv_triton.py:390-464).
//   3. score: grid (key tiles, B*Hkv).  Recomputes each logit, p = exp(l - lse)
//      clamped to [0,1] and optionally rounded to the input dtype, the weight
//      w = (p / (1 - p + eps))^2 and accumulates per key
//        SW = sum_m w, SB = sum_m w <v_j, y_m>, SC = sum_m w ||y_m||^2,
//      then score_j = (SW ||v_j||^2 - 2 SB + SC) / g: the reference's
//      termA - termB + termC (dropkv_triton.py:94-108), without clamping.
#include "common.cuh"

namespace dropkv {
namespace {

constexpr int TJ = 64;        // keys per tile
constexpr int MC = 32;        // query rows per chunk (8 threads per row)
constexpr int NT = 256;       // threads per CTA
constexpr int PST = TJ + 8;   // row stride of the p tile (bank-conflict free)
constexpr int MAX_SPLITS = 128;

template <typename T>
struct Vec {
  static constexpr int n = 16 / sizeof(T);
};

// Load rows [base, base+TJ) of one head's [Lk, D] matrix into smem as fp32
// (row stride D+1); rows past Lk are zero.
template <typename T, int D>
__device__ __forceinline__ void load_tile_f32(float* dst, const T* src_head, int base, int Lk) {
  constexpr int VE = Vec<T>::n;
  constexpr int CR = D / VE;
  constexpr int DP = D + 1;
  for (int c = threadIdx.x; c < TJ * CR; c += NT) {
    int row = c / CR;
    int col = (c % CR) * VE;
    int key = base + row;
    float* o = dst + row * DP + col;
    if (key < Lk) {
      uint4 raw = *reinterpret_cast<const uint4*>(src_head + (size_t)key * D + col);
      const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
      for (int i = 0; i < VE; ++i) o[i] = to_f<T>(e[i]);
    } else {
#pragma unroll
      for (int i = 0; i < VE; ++i) o[i] = 0.f;
    }
  }
}

// Query rows [m0, m0+MC) of head bh into smem (fp32, row stride D+1).
template <typename T, int D>
__device__ __forceinline__ void load_q_chunk(float* dst, const ScoreProblem& p, int b, int hkv,
                                             int m0) {
  constexpr int DP = D + 1;
  const T* q = reinterpret_cast<const T*>(p.q);
  for (int i = threadIdx.x; i < MC * D; i += NT) {
    int r = i / D, d = i % D;
    int m = m0 + r;
    float val = 0.f;
    if (m < p.M) {
      int qh = hkv * p.g + m / p.W;
      int qpos = p.Lq - p.W + m % p.W;
      val = to_f<T>(q[(int64_t)b * p.q_sb + (int64_t)qh * p.q_sh + (int64_t)qpos * p.q_ss +
                      (int64_t)d * p.q_sd]);
    }
    dst[r * DP + d] = val;
  }
}

template <typename T, int D>
__global__ void __launch_bounds__(NT) fwd_partial_kernel(ScoreProblem p, ScorePlan plan, float* ws) {
  constexpr int DP = D + 1;
  constexpr int DD = D / 8;
  extern __shared__ float sm[];
  float* qs = sm;
  float* ks = qs + MC * DP;
  float* vs = ks + TJ * DP;
  float* ps = vs + TJ * DP;

  const int s_idx = blockIdx.x;
  const int bh = blockIdx.y;
  const int b = bh / p.Hkv, hkv = bh % p.Hkv;
  const int tid = threadIdx.x;
  const int r = tid >> 3, sub = tid & 7;
  const T* kh = reinterpret_cast<const T*>(p.k) + (size_t)bh * p.kv_sh;
  const T* vh = reinterpret_cast<const T*>(p.v) + (size_t)bh * p.kv_sh;

  const int t_begin = s_idx * plan.tps;
  const int t_end = min(t_begin + plan.tps, plan.tiles);
  const float sqrt_d = sqrtf((float)D);

  float* part_m = ws + plan.off_pm / 4;
  float* part_s = ws + plan.off_ps / 4;
  float* part_y = ws + plan.off_py / 4;

  for (int m0 = 0; m0 < p.M; m0 += MC) {
    __syncthreads();
    load_q_chunk<T, D>(qs, p, b, hkv, m0);
    const int m = m0 + r;
    const bool row_ok = m < p.M;
    const int bound = p.Lk - p.W + (row_ok ? (m % p.W) : 0);
    float m_run = -INFINITY, s_run = 0.f;
    float acc[DD];
#pragma unroll
    for (int i = 0; i < DD; ++i) acc[i] = 0.f;

    for (int t = t_begin; t < t_end; ++t) {
      const int base = t * TJ;
      __syncthreads();
      load_tile_f32<T, D>(ks, kh, base, p.Lk);
      load_tile_f32<T, D>(vs, vh, base, p.Lk);
      __syncthreads();
      float sc[8];
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) sc[jj] = 0.f;
      for (int d = 0; d < D; ++d) {
        float qv = qs[r * DP + d];
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) sc[jj] = fmaf(qv, ks[(sub + 8 * jj) * DP + d], sc[jj]);
      }
      float tmax = -INFINITY;
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) {
        int key = base + sub + 8 * jj;
        bool ok = row_ok && key < p.Lk && key <= bound;
        sc[jj] = ok ? sc[jj] / sqrt_d : -INFINITY;
        tmax = fmaxf(tmax, sc[jj]);
      }
      tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 1));
      tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 2));
      tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 4));
      const float new_m = fmaxf(m_run, tmax);
      float alpha, psum = 0.f;
      if (new_m == -INFINITY) {
        alpha = 1.f;
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) ps[r * PST + sub + 8 * jj] = 0.f;
      } else {
        alpha = (m_run == -INFINITY) ? 0.f : expf(m_run - new_m);
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) {
          float e = (sc[jj] == -INFINITY) ? 0.f : expf(sc[jj] - new_m);
          psum += e;
          ps[r * PST + sub + 8 * jj] = e;
        }
      }
      psum += __shfl_xor_sync(0xffffffffu, psum, 1);
      psum += __shfl_xor_sync(0xffffffffu, psum, 2);
      psum += __shfl_xor_sync(0xffffffffu, psum, 4);
      s_run = s_run * alpha + psum;
      m_run = new_m;
#pragma unroll
      for (int i = 0; i < DD; ++i) acc[i] *= alpha;
      __syncthreads();
      for (int j = 0; j < TJ; ++j) {
        float pj = ps[r * PST + j];
        const float* vrow = vs + j * DP + sub;
#pragma unroll
        for (int i = 0; i < DD; ++i) acc[i] = fmaf(pj, vrow[8 * i], acc[i]);
      }
    }
    if (row_ok) {
      size_t prow = ((size_t)bh * plan.splits + s_idx) * p.M + m;
      if (sub == 0) {
        part_m[prow] = m_run;
        part_s[prow] = s_run;
      }
#pragma unroll
      for (int i = 0; i < DD; ++i) part_y[prow * D + sub + 8 * i] = acc[i];
    }
  }
}

// One CTA per head: merge split partials into lse, y (fp32) and ||y||^2.
__global__ void __launch_bounds__(NT) merge_kernel(ScoreProblem p, ScorePlan plan, float* ws) {
  __shared__ float c_sh[NT / 32][MAX_SPLITS];
  const int bh = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = plan.splits;
  const int D = p.D;
  const float* part_m = ws + plan.off_pm / 4;
  const float* part_s = ws + plan.off_ps / 4;
  const float* part_y = ws + plan.off_py / 4;
  float* lse = ws + plan.off_lse / 4;
  float* yn = ws + plan.off_yn / 4;
  float* y = ws + plan.off_y / 4;
  for (int m = warp; m < p.M; m += NT / 32) {
    float mx = -INFINITY;
    for (int s = lane; s < S; s += 32)
      mx = fmaxf(mx, part_m[((size_t)bh * S + s) * p.M + m]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float tot = 0.f;
    for (int s = lane; s < S; s += 32) {
      size_t pr = ((size_t)bh * S + s) * p.M + m;
      float ms = part_m[pr];
      float c = (ms == -INFINITY) ? 0.f : expf(ms - mx);
      c_sh[warp][s] = c;
      tot += c * part_s[pr];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
    __syncwarp();
    float n2 = 0.f;
    for (int d = lane; d < D; d += 32) {
      float a = 0.f;
      for (int s = 0; s < S; ++s) {
        float c = c_sh[warp][s];
        if (c != 0.f) a = fmaf(c, part_y[(((size_t)bh * S + s) * p.M + m) * D + d], a);
      }
      a = a / tot;
      y[((size_t)bh * p.M + m) * D + d] = a;
      n2 = fmaf(a, a, n2);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) n2 += __shfl_xor_sync(0xffffffffu, n2, o);
    if (lane == 0) {
      lse[(size_t)bh * p.M + m] = mx + logf(tot);
      yn[(size_t)bh * p.M + m] = n2;
    }
    __syncwarp();
  }
}

template <typename T, int D>
__global__ void __launch_bounds__(NT) score_kernel(ScoreProblem p, ScorePlan plan, const float* ws) {
  constexpr int DP = D + 1;
  extern __shared__ float sm[];
  float* ks = sm;
  float* vs = ks + TJ * DP;
  float* qs = vs + TJ * DP;
  float* ys = qs + MC * DP;
  float* redW = ys + MC * DP;        // [8 warps][TJ]
  float* redB = redW + 8 * TJ;
  float* redC = redB + 8 * TJ;
  float* lse_s = redC + 8 * TJ;      // [MC]
  float* yn_s = lse_s + MC;          // [MC]
  float* vn_s = yn_s + MC;           // [TJ]

  const int tile = blockIdx.x;
  const int bh = blockIdx.y;
  const int b = bh / p.Hkv, hkv = bh % p.Hkv;
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int r = tid >> 3, sub = tid & 7;
  const int base = tile * TJ;
  const T* kh = reinterpret_cast<const T*>(p.k) + (size_t)bh * p.kv_sh;
  const T* vh = reinterpret_cast<const T*>(p.v) + (size_t)bh * p.kv_sh;
  const float* lse = ws + plan.off_lse / 4;
  const float* yn = ws + plan.off_yn / 4;
  const float* yg = ws + plan.off_y / 4;
  const float sqrt_d = sqrtf((float)D);

  load_tile_f32<T, D>(ks, kh, base, p.Lk);
  load_tile_f32<T, D>(vs, vh, base, p.Lk);
  __syncthreads();
  if (tid < TJ) {
    float a = 0.f;
    for (int d = 0; d < D; ++d) a = fmaf(vs[tid * DP + d], vs[tid * DP + d], a);
    vn_s[tid] = a;
  }
  float accW = 0.f, accB = 0.f, accC = 0.f;  // owned by tid < TJ

  for (int m0 = 0; m0 < p.M; m0 += MC) {
    __syncthreads();
    load_q_chunk<T, D>(qs, p, b, hkv, m0);
    for (int i = tid; i < MC * D; i += NT) {
      int rr = i / D, d = i % D;
      int m = m0 + rr;
      ys[rr * DP + d] = (m < p.M) ? yg[((size_t)bh * p.M + m) * D + d] : 0.f;
    }
    if (tid < MC) {
      int m = m0 + tid;
      lse_s[tid] = (m < p.M) ? lse[(size_t)bh * p.M + m] : 0.f;
      yn_s[tid] = (m < p.M) ? yn[(size_t)bh * p.M + m] : 0.f;
    }
    __syncthreads();
    const int m = m0 + r;
    const bool row_ok = m < p.M;
    const int bound = p.Lk - p.W + (row_ok ? (m % p.W) : 0);
    float sc[8], dv[8];
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) { sc[jj] = 0.f; dv[jj] = 0.f; }
    for (int d = 0; d < D; ++d) {
      float qv = qs[r * DP + d];
      float yv = ys[r * DP + d];
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) {
        sc[jj] = fmaf(qv, ks[(sub + 8 * jj) * DP + d], sc[jj]);
        dv[jj] = fmaf(yv, vs[(sub + 8 * jj) * DP + d], dv[jj]);
      }
    }
    const float lse_m = lse_s[r];
    const float yn_m = yn_s[r];
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) {
      int key = base + sub + 8 * jj;
      bool ok = row_ok && key < p.Lk && key <= bound;
      float w = 0.f;
      if (ok) {
        float pr = expf(sc[jj] / sqrt_d - lse_m);
        pr = fminf(fmaxf(pr, 0.f), 1.f);
        pr = round_p(pr, p.round_mode);
        float ratio = pr / (1.f - pr + p.eps);
        w = ratio * ratio;
      }
      float cW = w, cB = w * dv[jj], cC = w * yn_m;
      // reduce over the 4 rows of this warp (lanes differing in bits 3,4)
      cW += __shfl_xor_sync(0xffffffffu, cW, 8);
      cB += __shfl_xor_sync(0xffffffffu, cB, 8);
      cC += __shfl_xor_sync(0xffffffffu, cC, 8);
      cW += __shfl_xor_sync(0xffffffffu, cW, 16);
      cB += __shfl_xor_sync(0xffffffffu, cB, 16);
      cC += __shfl_xor_sync(0xffffffffu, cC, 16);
      if (lane < 8) {
        redW[warp * TJ + sub + 8 * jj] = cW;
        redB[warp * TJ + sub + 8 * jj] = cB;
        redC[warp * TJ + sub + 8 * jj] = cC;
      }
    }
    __syncthreads();
    if (tid < TJ) {
#pragma unroll
      for (int w8 = 0; w8 < NT / 32; ++w8) {
        accW += redW[w8 * TJ + tid];
        accB += redB[w8 * TJ + tid];
        accC += redC[w8 * TJ + tid];
      }
    }
  }
  if (tid < TJ) {
    int key = base + tid;
    if (key < p.Lk) {
      float s = accW * vn_s[tid] - 2.f * accB + accC;
      p.scores[(size_t)bh * p.Lk + key] = s / (float)p.g;
    }
  }
}

template <typename T, int D>
size_t fwd_smem() { return sizeof(float) * ((size_t)MC * (D + 1) + 2 * (size_t)TJ * (D + 1) + (size_t)MC * PST); }
template <typename T, int D>
size_t score_smem() {
  return sizeof(float) * (2 * (size_t)TJ * (D + 1) + 2 * (size_t)MC * (D + 1) + 3 * 8 * TJ + 2 * MC + TJ);
}

template <typename T, int D>
int launch_typed(const ScoreProblem& p, const ScorePlan& plan, float* ws, cudaStream_t st) {
  size_t fs = fwd_smem<T, D>(), ss = score_smem<T, D>();
  static DeviceOnce attr_done;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_done.done(dev)) {
    if (cudaFuncSetAttribute(fwd_partial_kernel<T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)fs) !=
            cudaSuccess ||
        cudaFuncSetAttribute(score_kernel<T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ss) != cudaSuccess)
      return fail(DROPKV_ERR_CUDA, "cannot set shared memory sizes of the CUDA-core scorer");
    attr_done.mark(dev);
  }
  dim3 g1(plan.splits, plan.BH);
  fwd_partial_kernel<T, D><<<g1, NT, fs, st>>>(p, plan, ws);
  merge_kernel<<<plan.BH, NT, 0, st>>>(p, plan, ws);
  dim3 g3((p.Lk + TJ - 1) / TJ, plan.BH);
  score_kernel<T, D><<<g3, NT, ss, st>>>(p, plan, ws);
  return check_launch("scores_simt", 3);
}

template <typename T>
int launch_d(const ScoreProblem& p, const ScorePlan& plan, float* ws, cudaStream_t st) {
  switch (p.D) {
    case 32: return launch_typed<T, 32>(p, plan, ws, st);
    case 64: return launch_typed<T, 64>(p, plan, ws, st);
    case 128: return launch_typed<T, 128>(p, plan, ws, st);
    case 256: return launch_typed<T, 256>(p, plan, ws, st);
    default: return fail(DROPKV_ERR_UNSUPPORTED, "head_dim %d not supported (32, 64, 128, 256)", p.D);
  }
}

}  // namespace

int simt_max_splits() { return MAX_SPLITS; }
int simt_tile() { return TJ; }

int launch_scores_simt(const ScoreProblem& p, const ScorePlan& plan, void* ws, cudaStream_t st,
                       int dtype) {
  if (plan.tile != TJ) return fail(DROPKV_ERR_ARG, "internal: scorer plan tile mismatch");
  if (plan.splits > MAX_SPLITS) return fail(DROPKV_ERR_ARG, "internal: too many splits");
  float* w = reinterpret_cast<float*>(ws);
  switch (dtype) {
    case DROPKV_DTYPE_F32: return launch_d<float>(p, plan, w, st);
    case DROPKV_DTYPE_F16: return launch_d<__half>(p, plan, w, st);
    case DROPKV_DTYPE_BF16: return launch_d<__nv_bfloat16>(p, plan, w, st);
    default: return fail(DROPKV_ERR_ARG, "unknown dtype %d", dtype);
  }
}

}  // namespace dropkv
