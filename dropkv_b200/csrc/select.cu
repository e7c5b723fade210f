// Pool + protect + top-k + ascending sort of the kept positions, one CTA per
// (sequence, KV head) row.  Replaces dropkv_cache.py:464-475:
//
//   pooled = max_pool1d(scores, k, padding=k//2, stride=1)   (windows truncated)
//   pooled[-protect:] = amax(pooled) + 1
//   keep_idx = sort(topk(pooled, keep_len).indices)
//
// Selection is a radix select on order-preserving 32-bit keys (11/11/10-bit
// digits, 2048-bin shared-memory histograms) that finds the keep_len-th largest
// key T; the row is then compacted in index order keeping every key > T and the
// first (keep_len - #{key > T}) keys == T, i.e. ties go to the lower index.
// The output is therefore already sorted: no sort pass is needed.
#include "common.cuh"

namespace dropkv {
namespace {

constexpr int SNT = 1024;         // threads per CTA
constexpr int IPT = 4;            // items per thread in the compaction sweep

__device__ __forceinline__ int warp_incl_scan(int v, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int n = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += n;
  }
  return v;
}

// Block-wide exclusive scan of one int per thread; returns the exclusive prefix
// and writes the block total to *total.  `tmp` holds 33 ints.
__device__ __forceinline__ int block_excl_scan(int v, int* tmp, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nw = blockDim.x >> 5;
  int inc = warp_incl_scan(v, lane);
  if (lane == 31) tmp[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    int t = lane < nw ? tmp[lane] : 0;
    int ti = warp_incl_scan(t, lane);
    if (lane < nw) tmp[lane] = ti - t;  // exclusive warp offsets
    if (lane == 31) tmp[32] = ti;
  }
  __syncthreads();
  int res = tmp[warp] + inc - v;
  *total = tmp[32];
  __syncthreads();
  return res;
}

__device__ __forceinline__ float block_max(float v, float* tmp) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nw = blockDim.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  if (lane == 0) tmp[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float t = lane < nw ? tmp[lane] : -INFINITY;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t = fmaxf(t, __shfl_xor_sync(0xffffffffu, t, o));
    if (lane == 0) tmp[32] = t;
  }
  __syncthreads();
  float r = tmp[32];
  __syncthreads();
  return r;
}

__global__ void __launch_bounds__(SNT) select_row_kernel(const float* __restrict__ scores, int Lk,
                                                         int radius, int protect, int keep_len,
                                                         int64_t* __restrict__ keep_idx,
                                                         uint32_t* __restrict__ pooled_ws) {
  __shared__ uint32_t hist[2048];
  __shared__ int itmp[33];
  __shared__ float ftmp[33];
  __shared__ uint32_t sel_bin;
  __shared__ int sel_k;

  const int row = blockIdx.x;
  const int tid = threadIdx.x;
  const float* s = scores + (size_t)row * Lk;
  uint32_t* pw = pooled_ws + (size_t)row * Lk;

  // 1. sliding max (padding -inf == truncated window) and row max
  float lmax = -INFINITY;
  for (int j = tid; j < Lk; j += SNT) {
    int lo = max(0, j - radius), hi = min(Lk - 1, j + radius);
    float m = s[lo];
    for (int t = lo + 1; t <= hi; ++t) m = fmaxf(m, s[t]);
    pw[j] = __float_as_uint(m);
    lmax = fmaxf(lmax, m);
  }
  const float amax = block_max(lmax, ftmp);
  const float big = amax + 1.0f;
  const int pstart = Lk - protect;   // positions >= pstart are protected
  __syncthreads();

  // 2. radix select of the keep_len-th largest key
  uint32_t prefix = 0, pmask = 0;
  int k = keep_len;
  const int shifts[3] = {21, 10, 0};
  const int bits[3] = {11, 11, 10};
#pragma unroll
  for (int pass = 0; pass < 3; ++pass) {
    const int sh = shifts[pass];
    const int nb = 1 << bits[pass];
    const uint32_t dmask = (uint32_t)(nb - 1);
    for (int i = tid; i < 2048; i += SNT) hist[i] = 0;
    __syncthreads();
    for (int j = tid; j < Lk; j += SNT) {
      float v = (j >= pstart) ? big : __uint_as_float(pw[j]);
      uint32_t key = ordered_key(v);
      if ((key & pmask) == prefix) atomicAdd(&hist[(key >> sh) & dmask], 1u);
    }
    __syncthreads();
    // bins owned by this thread: 2*tid, 2*tid+1 (nb <= 2048); scan from the top
    const int b0 = 2 * tid, b1 = 2 * tid + 1;
    int h0 = b0 < nb ? (int)hist[b0] : 0;
    int h1 = b1 < nb ? (int)hist[b1] : 0;
    // suffix scan in descending thread order: above = #keys in bins > b1
    const int v = h0 + h1;
    int above;
    {
      const int lane = tid & 31, warp = tid >> 5;
      int inc = v;  // sum over lanes >= lane
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        int n = __shfl_down_sync(0xffffffffu, inc, o);
        if (lane + o < 32) inc += n;
      }
      if (lane == 0) itmp[warp] = inc;  // warp total
      __syncthreads();
      if (warp == 0) {
        const int nw = SNT / 32;
        int t = lane < nw ? itmp[lane] : 0;
        int si = t;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          int n = __shfl_down_sync(0xffffffffu, si, o);
          if (lane + o < 32) si += n;
        }
        if (lane < nw) itmp[lane] = si - t;  // keys in warps above this one
      }
      __syncthreads();
      above = itmp[warp] + inc - v;
      __syncthreads();
    }
    if (above < k && k <= above + h1) {
      sel_bin = (uint32_t)b1;
      sel_k = k - above;
    } else if (above + h1 < k && k <= above + h1 + h0) {
      sel_bin = (uint32_t)b0;
      sel_k = k - above - h1;
    }
    __syncthreads();
    prefix |= sel_bin << sh;
    pmask |= dmask << sh;
    k = sel_k;
    __syncthreads();
  }
  const uint32_t T = prefix;
  const int need_eq = k;  // keys == T to keep, in index order

  // 3. ordered compaction
  int out_base = 0, eq_base = 0;
  int64_t* out = keep_idx + (size_t)row * keep_len;
  for (int base = 0; base < Lk; base += SNT * IPT) {
    uint32_t keys[IPT];
    int ceq = 0;
#pragma unroll
    for (int i = 0; i < IPT; ++i) {
      int j = base + tid * IPT + i;
      if (j < Lk) {
        float v = (j >= pstart) ? big : __uint_as_float(pw[j]);
        keys[i] = ordered_key(v);
      } else {
        keys[i] = 0u;  // past the row end: excluded by the j < Lk tests below
      }
      ceq += (j < Lk && keys[i] == T) ? 1 : 0;
    }
    int eq_tot;
    int eq_before = block_excl_scan(ceq, itmp, &eq_tot) + eq_base;
    int keep_flags = 0, ck = 0;
#pragma unroll
    for (int i = 0; i < IPT; ++i) {
      int j = base + tid * IPT + i;
      bool kp = false;
      if (j < Lk) {
        if (keys[i] > T) kp = true;
        else if (keys[i] == T) {
          kp = eq_before < need_eq;
          ++eq_before;
        }
      }
      if (kp) { keep_flags |= 1 << i; ++ck; }
    }
    int k_tot;
    int pos = block_excl_scan(ck, itmp, &k_tot) + out_base;
#pragma unroll
    for (int i = 0; i < IPT; ++i) {
      if (keep_flags & (1 << i)) {
        if (pos < keep_len) out[pos] = base + tid * IPT + i;
        ++pos;
      }
    }
    out_base += k_tot;
    eq_base += eq_tot;
  }
}

}  // namespace

SelectPlan plan_select(int BH, int Lk) {
  SelectPlan p;
  p.off_keys = 0;
  p.bytes = align_up((size_t)BH * Lk * sizeof(uint32_t), 256);
  return p;
}

int launch_select(const float* scores, int BH, int Lk, int kernel_size, int protect, int keep_len,
                  int64_t* keep_idx, void* ws, cudaStream_t st) {
  uint32_t* pw = reinterpret_cast<uint32_t*>(ws);
  select_row_kernel<<<BH, SNT, 0, st>>>(scores, Lk, kernel_size / 2, protect, keep_len, keep_idx, pw);
  return check_launch("select");
}

}  // namespace dropkv
