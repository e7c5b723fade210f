// Cluster-parallel selection + compaction: pool, protect, top-k, ascending sort
// and the gather of the kept K/V rows in one launch (dropkv_cache.py:464-491).
//
// One thread-block cluster of CL CTAs per (sequence, KV head) row; CTA r of the
// cluster owns positions [r*chunk, (r+1)*chunk).  Everything stays in shared
// memory; the cluster cooperates through distributed shared memory:
//   1. pooled = sliding max over +-radius (halo read from global), row max by an
//      all-gather of the CTA maxima, protected tail := amax + 1;
//   2. radix select of the keep_len-th largest order-preserving key (11/11/10-bit
//      digits): per digit every CTA builds a 2048-bin histogram, CTA r sums bins
//      [r*B/CL, (r+1)*B/CL) over the cluster, finds the selected bin if it owns it
//      and publishes (bin, remaining k) to every CTA;
//   3. ordered compaction: per-CTA counts of keys > T and == T are exchanged, the
//      first (k - #{> T}) keys equal to T in index order are kept (ties to the
//      lower index), each CTA writes its slice of keep_idx in ascending order;
//   4. each CTA copies its kept K and V rows (16-byte vectors) to the outputs.
// No wait here is unbounded: cluster barriers are hardware barriers of
// co-scheduled CTAs.
#include <cooperative_groups.h>

#include <algorithm>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace dropkv {
namespace {

constexpr int SG_NT = 512;
constexpr int SG_MAXCL = 16;

__device__ __forceinline__ int sg_block_excl_scan(int v, int* tmp, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nw = blockDim.x >> 5;
  int inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int n = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += n;
  }
  if (lane == 31) tmp[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    int t = lane < nw ? tmp[lane] : 0;
    int ti = t;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int n = __shfl_up_sync(0xffffffffu, ti, o);
      if (lane >= o) ti += n;
    }
    if (lane < nw) tmp[lane] = ti - t;
    if (lane == 31) tmp[32] = ti;
  }
  __syncthreads();
  int res = tmp[warp] + inc - v;
  *total = tmp[32];
  __syncthreads();
  return res;
}

struct SgShared {  // static part of the shared memory
  uint32_t hist[2048];
  int itmp[33];
  float fmax_slot;
  int cnt_slot[4];          // published per-CTA values
  int sel_slot[2];          // selected bin, remaining k (written by the owner into every CTA)
  float ftmp[33];
};

template <typename VT>
__global__ void __launch_bounds__(SG_NT) select_gather_kernel(
    const float* __restrict__ scores, int Lk, int chunk, int radius, int protect, int keep_len,
    int64_t* __restrict__ keep_idx, const VT* __restrict__ kin, const VT* __restrict__ vin,
    VT* __restrict__ kout, VT* __restrict__ vout, int row_vecs) {
  cg::cluster_group cluster = cg::this_cluster();
  const int CL = (int)cluster.num_blocks();
  const int r = (int)cluster.block_rank();
  const int row = blockIdx.x / CL;
  const int tid = threadIdx.x;
  __shared__ SgShared S;
  extern __shared__ uint32_t dyn[];
  uint32_t* keys = dyn;                                 // [chunk]
  float* buf = reinterpret_cast<float*>(dyn + chunk);   // [chunk + 2 radius] scores; later kept list

  const int j0 = min(Lk, r * chunk), j1 = min(Lk, j0 + chunk);
  const int n = j1 - j0;
  const float* srow = scores + (size_t)row * Lk;

  // ---- 1. sliding max and row max -------------------------------------------
  const int h0 = max(0, j0 - radius), h1 = min(Lk, j1 + radius);
  for (int j = h0 + tid; j < h1; j += 8 * SG_NT) {  // 8 independent loads in flight per thread
    float v8[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int jj = j + u * SG_NT;
      v8[u] = (jj < h1) ? __ldg(srow + jj) : 0.f;
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int jj = j + u * SG_NT;
      if (jj < h1) buf[jj - h0] = v8[u];
    }
  }
  __syncthreads();
  float lmax = -INFINITY;
  for (int i = tid; i < n; i += SG_NT) {
    const int j = j0 + i;
    const int lo = max(0, j - radius), hi = min(Lk - 1, j + radius);
    float m = buf[lo - h0];
    for (int t = lo + 1; t <= hi; ++t) m = fmaxf(m, buf[t - h0]);
    keys[i] = __float_as_uint(m);
    lmax = fmaxf(lmax, m);
  }
  {
    const int lane = tid & 31, warp = tid >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) lmax = fmaxf(lmax, __shfl_xor_sync(0xffffffffu, lmax, o));
    if (lane == 0) S.ftmp[warp] = lmax;
    __syncthreads();
    if (tid == 0) {
      float m = S.ftmp[0];
      for (int w = 1; w < SG_NT / 32; ++w) m = fmaxf(m, S.ftmp[w]);
      S.fmax_slot = m;
    }
  }
  cluster.sync();
  float amax = -INFINITY;
  for (int c = 0; c < CL; ++c) amax = fmaxf(amax, *cluster.map_shared_rank(&S.fmax_slot, c));
  const float big = amax + 1.0f;
  const int pstart = Lk - protect;
  for (int i = tid; i < n; i += SG_NT) {
    const int j = j0 + i;
    keys[i] = ordered_key(j >= pstart ? big : __uint_as_float(keys[i]));
  }
  __syncthreads();

  // ---- 2. radix select over the cluster -------------------------------------
  uint32_t prefix = 0, pmask = 0;
  int k = keep_len;
#pragma unroll 1
  for (int pass = 0; pass < 3; ++pass) {
    const int sh = pass == 0 ? 21 : (pass == 1 ? 10 : 0);
    const int nb = pass == 2 ? 1024 : 2048;
    const uint32_t dmask = (uint32_t)(nb - 1);
    for (int i = tid; i < 2048; i += SG_NT) S.hist[i] = 0;
    __syncthreads();
    for (int i = tid; i < n; i += SG_NT) {
      const uint32_t key = keys[i];
      if ((key & pmask) == prefix) atomicAdd(&S.hist[(key >> sh) & dmask], 1u);
    }
    cluster.sync();  // every histogram complete
    // reduce-scatter: this CTA owns bins [b_lo, b_hi), 4 contiguous bins per thread
    const int per = (nb + CL - 1) / CL;
    const int b_lo = min(nb, r * per), b_hi = min(nb, b_lo + per);
    const int tb0 = b_lo + tid * 4;
    int cnt[4];
    int my_sum = 0;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int bb = tb0 + u;
      cnt[u] = 0;
      if (bb < b_hi) {
        uint32_t sum = 0;
        for (int c = 0; c < CL; ++c) sum += cluster.map_shared_rank(S.hist, c)[bb];
        cnt[u] = (int)sum;
        my_sum += (int)sum;
      }
    }
    int blk_total;
    const int excl = sg_block_excl_scan(my_sum, S.itmp, &blk_total);
    if (tid == 0) S.cnt_slot[0] = blk_total;
    cluster.sync();  // range totals published; remote histogram reads finished
    int acc = blk_total - (excl + my_sum);  // keys in this CTA's bins above mine
    for (int c = r + 1; c < CL; ++c) acc += cluster.map_shared_rank(S.cnt_slot, c)[0];
#pragma unroll
    for (int u = 3; u >= 0; --u) {
      const int bb = tb0 + u;
      if (bb < b_hi) {
        if (acc < k && k <= acc + cnt[u]) {
          for (int c = 0; c < CL; ++c) {
            int* sl = cluster.map_shared_rank(S.sel_slot, c);
            sl[0] = bb;
            sl[1] = k - acc;
          }
        }
        acc += cnt[u];
      }
    }
    cluster.sync();  // selection published
    prefix |= ((uint32_t)S.sel_slot[0]) << sh;
    pmask |= dmask << sh;
    k = S.sel_slot[1];
    cluster.sync();  // slots may be rewritten next pass only after everyone read them
  }
  const uint32_t T = prefix;
  const int need_eq = k;

  // ---- 3. ordered compaction -------------------------------------------------
  int cgt = 0, ceq = 0;
  for (int i = tid; i < n; i += SG_NT) {
    const uint32_t key = keys[i];
    cgt += key > T;
    ceq += key == T;
  }
  int tot_gt, tot_eq;
  (void)sg_block_excl_scan(cgt, S.itmp, &tot_gt);
  (void)sg_block_excl_scan(ceq, S.itmp, &tot_eq);
  if (tid == 0) {
    S.cnt_slot[1] = tot_gt;
    S.cnt_slot[2] = tot_eq;
  }
  cluster.sync();
  int eq_before = 0, out_before = 0;
  for (int c = 0; c < r; ++c) {
    const int* sl = cluster.map_shared_rank(S.cnt_slot, c);
    const int g = sl[1], e = sl[2];
    const int keep_e = max(0, min(e, need_eq - eq_before));
    out_before += g + keep_e;
    eq_before += e;
  }
  int* kept = reinterpret_cast<int*>(buf);  // [<= chunk] kept positions, ascending
  int n_kept = 0, eq_run = eq_before;
  for (int base = 0; base < n; base += SG_NT * 4) {
    uint32_t kk[4];
    int neq = 0;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = base + tid * 4 + u;
      kk[u] = (i < n) ? keys[i] : 0u;
      neq += (i < n && kk[u] == T);
    }
    int eq_tot;
    int eqb = sg_block_excl_scan(neq, S.itmp, &eq_tot) + eq_run;
    int flags = 0, nk = 0;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = base + tid * 4 + u;
      bool kp = false;
      if (i < n) {
        if (kk[u] > T) kp = true;
        else if (kk[u] == T) {
          kp = eqb < need_eq;
          ++eqb;
        }
      }
      if (kp) { flags |= 1 << u; ++nk; }
    }
    int k_tot;
    int pos = sg_block_excl_scan(nk, S.itmp, &k_tot) + n_kept;
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (flags & (1 << u)) kept[pos++] = j0 + base + tid * 4 + u;
    n_kept += k_tot;
    eq_run += eq_tot;
    __syncthreads();
  }
  __syncthreads();
  int64_t* orow = keep_idx + (size_t)row * keep_len;
  for (int i = tid; i < n_kept; i += SG_NT)
    if (out_before + i < keep_len) orow[out_before + i] = kept[i];

  // ---- 4. gather the kept rows (select-only calls pass no K/V) ---------------
  if (kin == nullptr) {
    cluster.sync();
    return;
  }
  const VT* kr = kin + (size_t)row * Lk * row_vecs;
  const VT* vr = vin + (size_t)row * Lk * row_vecs;
  VT* ko = kout + (size_t)row * keep_len * row_vecs;
  VT* vo = vout + (size_t)row * keep_len * row_vecs;
  const int total = n_kept * row_vecs;
  for (int c0 = tid; c0 < total; c0 += 4 * SG_NT) {  // 8 independent loads in flight per thread
    VT kv[4], vv[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int c = c0 + u * SG_NT;
      if (c < total) {
        const int i = c / row_vecs, col = c - i * row_vecs;
        const size_t src = (size_t)kept[i] * row_vecs + col;
        kv[u] = kr[src];
        vv[u] = vr[src];
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int c = c0 + u * SG_NT;
      if (c < total) {
        const int i = c / row_vecs, col = c - i * row_vecs;
        const int o = out_before + i;
        if (o < keep_len) {
          ko[(size_t)o * row_vecs + col] = kv[u];
          vo[(size_t)o * row_vecs + col] = vv[u];
        }
      }
    }
  }
  cluster.sync();  // keep remote shared memory alive until every CTA is done with it
}

}  // namespace

// Cluster size and chunk for a row of Lk positions; 0 if the row does not fit.
static int sg_cluster_for(int Lk, int radius, int* chunk_out, size_t* smem_out) {
  int cl = 1;
  while (cl < SG_MAXCL && (Lk + cl - 1) / cl > 4096) cl *= 2;
  const int chunk = (Lk + cl - 1) / cl;
  const size_t smem = (size_t)chunk * 4 + ((size_t)chunk + 2 * (size_t)radius) * 4;
  if (smem + sizeof(SgShared) > 227 * 1024) return 0;
  *chunk_out = chunk;
  *smem_out = smem;
  return cl;
}

bool select_gather_supported(int Lk, int kernel_size) {
  int chunk;
  size_t smem;
  return sg_cluster_for(Lk, kernel_size / 2, &chunk, &smem) > 0;
}

template <typename VT>
static int launch_sg(const float* scores, int BH, int Lk, int kernel_size, int protect, int keep_len,
                     int64_t* keep_idx, const void* k, const void* v, int row_bytes, void* ko, void* vo,
                     cudaStream_t st) {
  int chunk;
  size_t smem;
  const int cl = sg_cluster_for(Lk, kernel_size / 2, &chunk, &smem);
  if (!cl) return fail(DROPKV_ERR_UNSUPPORTED, "row of %d positions too long for the cluster select", Lk);
  auto kern = select_gather_kernel<VT>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (cl > 8) cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(BH * cl);
  cfg.blockDim = dim3(SG_NT);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cl;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const int vecs = row_bytes / (int)sizeof(VT);
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, scores, Lk, chunk, kernel_size / 2, protect, keep_len, keep_idx,
                                     reinterpret_cast<const VT*>(k), reinterpret_cast<const VT*>(v),
                                     reinterpret_cast<VT*>(ko), reinterpret_cast<VT*>(vo), vecs);
  if (e != cudaSuccess) return fail(DROPKV_ERR_CUDA, "select_gather launch: %s", cudaGetErrorString(e));
  return check_launch("select_gather");
}

int launch_select_gather(const float* scores, int BH, int Lk, int kernel_size, int protect, int keep_len,
                         int64_t* keep_idx, const void* k, const void* v, int elem_bytes, int D, void* ko,
                         void* vo, cudaStream_t st) {
  const int row_bytes = D * elem_bytes;
  auto al = [](const void* p, int a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; };
  if (row_bytes % 16 == 0 && al(k, 16) && al(v, 16) && al(ko, 16) && al(vo, 16))
    return launch_sg<uint4>(scores, BH, Lk, kernel_size, protect, keep_len, keep_idx, k, v, row_bytes, ko, vo, st);
  if (row_bytes % 4 == 0 && al(k, 4) && al(v, 4) && al(ko, 4) && al(vo, 4))
    return launch_sg<uint32_t>(scores, BH, Lk, kernel_size, protect, keep_len, keep_idx, k, v, row_bytes, ko, vo, st);
  return launch_sg<uint16_t>(scores, BH, Lk, kernel_size, protect, keep_len, keep_idx, k, v, row_bytes, ko, vo, st);
}

}  // namespace dropkv
