// Decode attention over the (compressed) KV cache: for every sequence b and query
// head h, O[b, h, i, :] = softmax(scale * Q[b, h, i, :] K[b, h / g, :L, :]^T) V[b, h / g, :L, :]
// with the Lq query rows tail-aligned to the keys (row i sees keys j <= L - Lq + i),
// which is what the model's attention computes over the cache DropKVCache.update
// returns (dropkv_cache.py:609-617 append the token, the model's SDPA attends).
//
// With one to a few query rows per KV head the work is a matrix-vector product per
// key: HBM-bound, no tensor-core tile to fill. One thread-block cluster of CL CTAs
// per (sequence, KV head, block of up to MR query rows); CTA r takes a contiguous
// range of keys. In each CTA a producer warp streams chunks of KC keys of K and V
// (contiguous rows) into a 4-stage shared-memory ring with bulk copies on
// mbarriers, and CW compute warps consume them (4 warps and 32-key chunks: small
// CTAs, so that several share an SM and the clusters of a launch are resident
// together): a key row is read by D/8 lanes,
// 16 bytes each, every lane keeping the running max, sum and output of its 8
// columns for each query row (softmax in base 2). The CTAs' partials (max, sum,
// output) are merged through distributed shared memory in CTA order, each CTA
// writing a slice of O. Every wait is bounded; a wait that gives up sets a bit in
// the status word (the first 4 bytes of the workspace) and the kernel finishes.
#include <cooperative_groups.h>

#include <algorithm>
#include <type_traits>

#include "tc_common.cuh"

namespace cg = cooperative_groups;

namespace dropkv {
namespace {

constexpr int DA_ST = 4;                 // ring stages
constexpr int DA_MAXCL = 16;
constexpr uint64_t DA_WAIT_NS = 1000000000ull;

struct DaArgs {
  const void* q;
  int64_t q_sb, q_sh, q_ss, q_sd;
  const void* k;
  const void* v;
  int64_t kv_sb, kv_sh;  // element strides of a sequence and a KV head; rows of D contiguous
  int Hq, Hkv, g, Lq, L;
  int M;                 // g * Lq query rows per (b, KV head)
  int chunk;             // keys per CTA (a multiple of the kernel's KC)
  float scale_log2;      // scale * log2(e)
  int* status;
  void* out;             // [B, Hq, Lq, D]
};

// compute warps and keys per stage for MR query rows per CTA
template <int MR>
struct DaCfg {
  static constexpr int CW = 4;
  static constexpr int KC = 32;
  static constexpr int NT = 32 * (CW + 1);  // + the producer warp
};

template <int D, int MR, int EB>
struct DaLay {
  static constexpr int CW = DaCfg<MR>::CW, KC = DaCfg<MR>::KC;
  static constexpr int HALF = KC * D * EB;               // K (or V) rows of a stage
  static constexpr int STAGE = 2 * HALF;
  static constexpr int RING = 0;
  static constexpr int WACC = RING;                      // float [CW][MR][D], in the ring once drained
  static_assert(CW * MR * D * 4 <= DA_ST * STAGE, "warp partials fit the ring");
  static constexpr int QS = RING + DA_ST * STAGE;        // float [MR][D]
  static constexpr int WML = QS + MR * D * 4;            // float [CW][MR][2]
  static constexpr int PART = WML + CW * MR * 2 * 4;     // float [MR][D + 2]: this CTA's partial
  static constexpr int BND = PART + MR * (D + 2) * 4;    // int [MR]
  static constexpr int BAR = (BND + MR * 4 + 7) & ~7;    // full[DA_ST], empty[DA_ST]
  static constexpr int BYTES = BAR + 2 * DA_ST * 8;
};

template <typename T>
__device__ __forceinline__ void unpack8(const uint4& r, float* f) {
  const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if constexpr (std::is_same<T, __nv_bfloat16>::value) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    } else {
      const float2 x = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      f[2 * i] = x.x;
      f[2 * i + 1] = x.y;
    }
  }
}

template <typename T>
__device__ __forceinline__ T from_f(float x);
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <>
__device__ __forceinline__ __half from_f<__half>(float x) { return __float2half_rn(x); }

__device__ __forceinline__ float ex2(float x) {  // 2^x, hardware approximation; 2^-inf = 0
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <int NTH>
__device__ __forceinline__ void compute_sync() {  // the compute warps only
  asm volatile("bar.sync 1, %0;" ::"r"(NTH) : "memory");
}

template <typename T, int D, int MR>
__global__ void __launch_bounds__(DaCfg<MR>::NT, 1) decode_attn_kernel(DaArgs a) {
  using Ly = DaLay<D, MR, (int)sizeof(T)>;
  constexpr int DA_CW = DaCfg<MR>::CW, DA_KC = DaCfg<MR>::KC, DA_NT = DaCfg<MR>::NT;
  constexpr int LPK = D / 8;           // lanes per key row
  constexpr int KPW = 32 / LPK;        // keys per warp and load
  constexpr int KPWS = DA_KC / DA_CW;  // keys per warp and stage
  constexpr int U = KPWS / KPW;        // loads per warp and stage
  static_assert(U >= 1 && KPWS % KPW == 0, "whole loads per warp");
  extern __shared__ __align__(128) uint8_t smem[];
  cg::cluster_group cluster = cg::this_cluster();
  const int CL = (int)cluster.num_blocks(), cr = (int)cluster.block_rank();
  const int bh = blockIdx.y, rb = blockIdx.z;
  const int b = bh / a.Hkv, hkv = bh % a.Hkv;
  const int m0 = rb * MR, mr = min(MR, a.M - m0);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float* qs = reinterpret_cast<float*>(smem + Ly::QS);
  float* wacc = reinterpret_cast<float*>(smem + Ly::WACC);
  float* wml = reinterpret_cast<float*>(smem + Ly::WML);
  float* part = reinterpret_cast<float*>(smem + Ly::PART);
  int* bnd = reinterpret_cast<int*>(smem + Ly::BND);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Ly::BAR);
  uint64_t* empty = full + DA_ST;
  const int s0 = min(a.L, cr * a.chunk), s1 = min(a.L, s0 + a.chunk);
  const int nch = (s1 - s0 + DA_KC - 1) / DA_KC;  // stages of this CTA's keys
  const T* kb = reinterpret_cast<const T*>(a.k) + b * a.kv_sb + hkv * a.kv_sh;
  const T* vb = reinterpret_cast<const T*>(a.v) + b * a.kv_sb + hkv * a.kv_sh;

  if (tid == 0) {
    for (int st = 0; st < DA_ST; ++st) {
      tc::mbar_init(&full[st], 1);
      tc::mbar_init(&empty[st], DA_CW);
    }
    tc::fence_mbar_init();
  }
  __syncthreads();

  if (warp == DA_CW) {
    // ---- producer: K and V rows of each chunk of keys into the ring ----------
    if (lane == 0) {
      int c = 0;
      for (; c < nch; ++c) {
        const int st = c % DA_ST;
        if (c >= DA_ST && !tc::mbar_wait(&empty[st], ((c / DA_ST) - 1) & 1, DA_WAIT_NS)) {
          atomicOr(a.status, 1);
          break;
        }
        const int j0 = s0 + c * DA_KC, nk = min(DA_KC, s1 - j0);
        const uint32_t bytes = (uint32_t)(nk * D * (int)sizeof(T));
        tc::mbar_arrive_expect_tx(&full[st], 2 * bytes);
        tc::bulk_load(smem + Ly::RING + st * Ly::STAGE, kb + (int64_t)j0 * D, bytes, &full[st]);
        tc::bulk_load(smem + Ly::RING + st * Ly::STAGE + Ly::HALF, vb + (int64_t)j0 * D, bytes, &full[st]);
      }
      // the CTA stays alive until every issued copy has landed
      for (int j = max(0, c - DA_ST); j < c; ++j)
        if (!tc::mbar_wait(&full[j % DA_ST], (j / DA_ST) & 1, DA_WAIT_NS)) atomicOr(a.status, 4);
    }
  } else {
    // ---- compute warps --------------------------------------------------------
    // query rows m0 .. m0 + mr - 1 of the group: row m is head hkv * g + m / Lq at
    // query position m % Lq; pre-scaled so that logits come out in base 2
    const T* qp = reinterpret_cast<const T*>(a.q);
    for (int i = tid; i < MR * D; i += DA_CW * 32) {
      const int rr = i / D, d = i % D, m = m0 + rr;
      float x = 0.f;
      if (rr < mr) {
        const int h = hkv * a.g + m / a.Lq, qi = m % a.Lq;
        x = to_f(qp[b * a.q_sb + h * a.q_sh + qi * a.q_ss + d * a.q_sd]) * a.scale_log2;
      }
      qs[rr * D + d] = x;
    }
    if (tid < MR) bnd[tid] = (tid < mr) ? a.L - a.Lq + (m0 + tid) % a.Lq : -1;
    compute_sync<DA_CW * 32>();
    const int dl = (lane % LPK) * 8;  // this lane's 8 columns
    float qr[MR][8];
#pragma unroll
    for (int rr = 0; rr < MR; ++rr)
#pragma unroll
      for (int e = 0; e < 8; ++e) qr[rr][e] = qs[rr * D + dl + e];
    int bl[MR];
#pragma unroll
    for (int rr = 0; rr < MR; ++rr) bl[rr] = bnd[rr];
    float mrun[MR], lrun[MR], acc[MR][8];
#pragma unroll
    for (int rr = 0; rr < MR; ++rr) {
      mrun[rr] = -INFINITY;
      lrun[rr] = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[rr][e] = 0.f;
    }
    for (int c = 0; c < nch; ++c) {
      const int st = c % DA_ST;
      if (!tc::mbar_wait(&full[st], (c / DA_ST) & 1, DA_WAIT_NS)) {
        atomicOr(a.status, 2);
        break;
      }
      const T* ks = reinterpret_cast<const T*>(smem + Ly::RING + st * Ly::STAGE);
      const T* vs = reinterpret_cast<const T*>(smem + Ly::RING + st * Ly::STAGE + Ly::HALF);
      const int j0 = s0 + c * DA_KC;
      uint4 kr[U], vr[U];
      int jj[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int kk = warp * KPWS + u * KPW + lane / LPK;
        jj[u] = j0 + kk;
        if (jj[u] < s1) {
          kr[u] = *reinterpret_cast<const uint4*>(ks + kk * D + dl);
          vr[u] = *reinterpret_cast<const uint4*>(vs + kk * D + dl);
        } else {  // past this CTA's keys: the slot holds stale rows
          kr[u] = make_uint4(0u, 0u, 0u, 0u);
          vr[u] = kr[u];
        }
      }
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&empty[st]);  // this warp is done with the stage
      float s[U][MR];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        float kf[8];
        unpack8<T>(kr[u], kf);
#pragma unroll
        for (int rr = 0; rr < MR; ++rr) {
          float t = 0.f;
#pragma unroll
          for (int e = 0; e < 8; ++e) t = fmaf(qr[rr][e], kf[e], t);
          s[u][rr] = t;
        }
      }
      // full dot products: sum over the LPK lanes of each key
#pragma unroll
      for (int o = LPK / 2; o >= 1; o >>= 1)
#pragma unroll
        for (int u = 0; u < U; ++u)
#pragma unroll
          for (int rr = 0; rr < MR; ++rr) s[u][rr] += __shfl_xor_sync(0xffffffffu, s[u][rr], o);
#pragma unroll
      for (int rr = 0; rr < MR; ++rr) {
        float cm = -INFINITY;
#pragma unroll
        for (int u = 0; u < U; ++u) {
          if (jj[u] >= s1 || jj[u] > bl[rr]) s[u][rr] = -INFINITY;
          cm = fmaxf(cm, s[u][rr]);
        }
#pragma unroll
        for (int o = LPK; o < 32; o <<= 1) cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, o));
        const float mn = fmaxf(mrun[rr], cm);
        if (mn == -INFINITY) continue;  // nothing visible to this row yet (warp-uniform)
        const float sc = ex2(mrun[rr] - mn);
        mrun[rr] = mn;
        lrun[rr] *= sc;
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[rr][e] *= sc;
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const float p = ex2(s[u][rr] - mn);
          if (lane % LPK == 0) lrun[rr] += p;  // one lane per key counts it
          float vf[8];
          unpack8<T>(vr[u], vf);
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[rr][e] = fmaf(p, vf[e], acc[rr][e]);
        }
      }
    }
    // sum over the warp's keys (lanes with the same columns), then over the warps;
    // the ring is free once every warp is past its last stage
    compute_sync<DA_CW * 32>();
#pragma unroll
    for (int rr = 0; rr < MR; ++rr) {
#pragma unroll
      for (int o = LPK; o < 32; o <<= 1) {
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[rr][e] += __shfl_xor_sync(0xffffffffu, acc[rr][e], o);
      }
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) lrun[rr] += __shfl_xor_sync(0xffffffffu, lrun[rr], o);
      if (lane < LPK) {
#pragma unroll
        for (int e = 0; e < 8; ++e) wacc[(warp * MR + rr) * D + dl + e] = acc[rr][e];
      }
      if (lane == 0) {
        wml[(warp * MR + rr) * 2] = mrun[rr];
        wml[(warp * MR + rr) * 2 + 1] = lrun[rr];
      }
    }
    compute_sync<DA_CW * 32>();
    // this CTA's partial: max-rescaled sum of the warps'
    for (int i = tid; i < MR * D; i += DA_CW * 32) {
      const int rr = i / D, d = i % D;
      float mx = -INFINITY;
#pragma unroll
      for (int w = 0; w < DA_CW; ++w) mx = fmaxf(mx, wml[(w * MR + rr) * 2]);
      float o = 0.f, l = 0.f;
      if (mx != -INFINITY) {
#pragma unroll
        for (int w = 0; w < DA_CW; ++w) {
          const float f = ex2(wml[(w * MR + rr) * 2] - mx);
          o = fmaf(f, wacc[(w * MR + rr) * D + d], o);
          l = fmaf(f, wml[(w * MR + rr) * 2 + 1], l);
        }
      }
      part[rr * (D + 2) + d] = o;
      if (d == 0) {
        part[rr * (D + 2) + D] = mx;
        part[rr * (D + 2) + D + 1] = l;
      }
    }
  }
  cluster.sync();  // every CTA's partial is complete
  // ---- merge in CTA order: this CTA writes elements [e0, e1) of the mr x D block --
  const int E = mr * D;
  const int e0 = (int)(((long long)cr * E) / CL), e1 = (int)(((long long)(cr + 1) * E) / CL);
  T* op = reinterpret_cast<T*>(a.out);
  for (int e = e0 + tid; e < e1; e += DA_NT) {
    const int rr = e / D, d = e % D;
    float mx = -INFINITY;
    for (int c2 = 0; c2 < CL; ++c2) mx = fmaxf(mx, cluster.map_shared_rank(part, c2)[rr * (D + 2) + D]);
    float o = 0.f, l = 0.f;
    if (mx != -INFINITY) {
      for (int c2 = 0; c2 < CL; ++c2) {
        const float* pr = cluster.map_shared_rank(part, c2) + rr * (D + 2);
        const float ms = pr[D];
        if (ms == -INFINITY) continue;
        const float f = ex2(ms - mx);
        o = fmaf(f, pr[d], o);
        l = fmaf(f, pr[D + 1], l);
      }
    }
    const int m = m0 + rr, h = hkv * a.g + m / a.Lq, qi = m % a.Lq;
    op[(((size_t)b * a.Hq + h) * a.Lq + qi) * D + d] = from_f<T>(l > 0.f ? o / l : 0.f);
  }
  cluster.sync();  // keep this CTA's partial alive until the cluster has read it
}

using DaKernel = void (*)(DaArgs);

template <typename T, int D>
DaKernel pick_da(int mr, int* smem) {
  constexpr int EB = (int)sizeof(T);
  switch (mr) {
    case 1: *smem = DaLay<D, 1, EB>::BYTES; return decode_attn_kernel<T, D, 1>;
    case 2: *smem = DaLay<D, 2, EB>::BYTES; return decode_attn_kernel<T, D, 2>;
    case 4: *smem = DaLay<D, 4, EB>::BYTES; return decode_attn_kernel<T, D, 4>;
    default: *smem = DaLay<D, 8, EB>::BYTES; return decode_attn_kernel<T, D, 8>;
  }
}

int da_threads(int mr) { return mr <= 4 ? DaCfg<4>::NT : DaCfg<8>::NT; }
int da_keys_per_stage(int mr) { return mr <= 4 ? DaCfg<4>::KC : DaCfg<8>::KC; }

// Clusters of `cl` CTAs that can be resident at once (a cluster must fit in one
// GPC, and GPCs differ in size), cached per device, kernel variant and size.
int da_active_clusters(DaKernel kern, int var, int cl, int threads, int smem) {
  static std::atomic<int> cache[16][DA_MAXCL + 1][16];  // zero: not queried yet
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 16) {
    const int c = cache[var][cl][dev].load(std::memory_order_relaxed);
    if (c > 0) return c;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(cl);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cl;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n < 1) {
    cudaGetLastError();
    return 1 << 20;
  }
  if (dev >= 0 && dev < 16) cache[var][cl][dev].store(n, std::memory_order_relaxed);
  return n;
}

}  // namespace

size_t decode_attention_workspace_size(int, int, int, int, int, int) { return 256; }  // the status word

int launch_decode_attention(const void* q, int64_t q_sb, int64_t q_sh, int64_t q_ss, int64_t q_sd, int Lq,
                            const void* k, const void* v, int64_t kv_sb, int64_t kv_sh, int dtype, int B, int Hq,
                            int Hkv, int L, int D, float scale, void* out, void* ws, cudaStream_t st) {
  int dev = 0;
  cudaGetDevice(&dev);
  DaArgs a;
  a.q = q;
  a.q_sb = q_sb;
  a.q_sh = q_sh;
  a.q_ss = q_ss;
  a.q_sd = q_sd;
  a.k = k;
  a.v = v;
  a.kv_sb = kv_sb;
  a.kv_sh = kv_sh;
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.g = Hq / Hkv;
  a.Lq = Lq;
  a.L = L;
  a.M = a.g * Lq;
  const int mr = a.M <= 1 ? 1 : (a.M <= 2 ? 2 : (a.M <= 4 ? 4 : 8));
  const int nrb = (a.M + mr - 1) / mr;
  int smem = 0, var;
  DaKernel kern;
  if (dtype == DROPKV_DTYPE_BF16) {
    kern = D == 128 ? pick_da<__nv_bfloat16, 128>(mr, &smem) : pick_da<__nv_bfloat16, 64>(mr, &smem);
    var = D == 128 ? 0 : 4;
  } else {
    kern = D == 128 ? pick_da<__half, 128>(mr, &smem) : pick_da<__half, 64>(mr, &smem);
    var = D == 128 ? 8 : 12;
  }
  var += mr == 1 ? 0 : (mr == 2 ? 1 : (mr == 4 ? 2 : 3));
  static DeviceOnce done[16];  // attributes set, per variant and device
  if (!done[var].done(dev)) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess ||
        cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)
      return fail(DROPKV_ERR_CUDA, "cannot set decode attention kernel attributes");
    done[var].mark(dev);
  }
  // CTAs per cluster: the size that finishes soonest, counting the waves the
  // launch's clusters need and the key stages each CTA streams; at most 16
  const int rows = B * Hkv * nrb;
  const int kc = da_keys_per_stage(mr), threads = da_threads(mr);
  int cl = 1, chunk = ((L + kc - 1) / kc) * kc;
  double best = 1e30;
  for (int c = std::min(DA_MAXCL, (L + kc - 1) / kc); c >= 1; c /= 2) {
    int ch = (L + c - 1) / c;
    ch = ((ch + kc - 1) / kc) * kc;
    const int cc = (L + ch - 1) / ch;  // every CTA gets keys
    const int act = da_active_clusters(kern, var, cc, threads, smem);
    const double t = (double)((rows + act - 1) / act) * (ch / kc + 2);  // + merge and launch, in stages
    if (t < best - 1e-9) {
      best = t;
      cl = cc;
      chunk = ch;
    }
  }
  a.chunk = chunk;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.status = reinterpret_cast<int*>(ws);
  a.out = out;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(cl, B * Hkv, nrb);
  cfg.blockDim = dim3(da_threads(mr));
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cl;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a);
  if (e != cudaSuccess) return fail(DROPKV_ERR_CUDA, "decode attention launch: %s", cudaGetErrorString(e));
  return check_launch("decode_attention");
}

}  // namespace dropkv
