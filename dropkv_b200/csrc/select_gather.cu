// Cluster-parallel selection: pool, protect, top-k and ascending sort of the kept
// positions (dropkv_cache.py:464-475) in one launch; the kept K/V rows are then
// copied by the gather kernel, which spreads over the whole GPU.
//
// One thread-block cluster of CL CTAs per (sequence, KV head) row; CTA r of the
// cluster owns positions [r*chunk, (r+1)*chunk); each of its threads owns a run of
// consecutive positions and keeps their keys in registers for the whole kernel.
// The cluster cooperates through distributed shared memory:
//   1. pooled = sliding max over +-radius (the score window with its halo staged
//      in shared memory; max by doubling spans in registers), the CTA's maximum
//      is published;
//   2. radix select of the keep_len-th largest order-preserving key (11/11/10-bit
//      digits), one cluster barrier per digit: every CTA builds its histogram in
//      its own shared memory and adds the non-zero bins into their owner's copy
//      (CTA r owns bins [r*nb/CL, (r+1)*nb/CL), a separate array per digit, so
//      no barrier is needed before the next digit's adds); after the barrier
//      every CTA reads all reduced bins back and finds the selected bin itself.
//      In the first digit the row maximum is formed from the published CTA
//      maxima and the protected tail (value amax + 1, dropkv_cache.py:465-467)
//      is added to its bin by every CTA on read-back; from then on protected
//      positions carry that key. The keys matching the first digit form a
//      candidate list that the later digits scan instead of the whole chunk;
//   3. ordered compaction: one block scan of the per-thread counts of keys > T
//      and == T ranks every position; CTA totals are exchanged; the first
//      (k - #{> T}) keys equal to T in index order are kept (ties to the lower
//      index) and written to keep_idx in ascending order.
// CTAs of 512 threads: with up to 16 positions per thread two of them fit on an
// SM, so launches with many rows keep all their clusters resident. No wait here is
// unbounded: cluster barriers are hardware barriers of co-scheduled CTAs.
#include <cooperative_groups.h>

#include <algorithm>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace dropkv {
namespace {

constexpr int SG_NT = 512;  // 16 warps
constexpr int SG_NW = SG_NT / 32;
constexpr int SG_MAXCL = 16;

__device__ __forceinline__ int sg_block_excl_scan(int v, int* tmp, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int n = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += n;
  }
  if (lane == 31) tmp[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    int t = lane < SG_NW ? tmp[lane] : 0;
    int ti = t;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int n = __shfl_up_sync(0xffffffffu, ti, o);
      if (lane >= o) ti += n;
    }
    if (lane < SG_NW) tmp[lane] = ti - t;
    if (lane == 31) tmp[32] = ti;
  }
  __syncthreads();
  int res = tmp[warp] + inc - v;
  *total = tmp[32];
  __syncthreads();
  return res;
}

// Each thread owns KPT consecutive positions of its CTA's chunk (a chunk holds at
// most SG_NT * KPT positions) and keeps their keys in registers. The score window
// is staged in shared memory with one padding word after every KPT words, so that
// a warp reading its lanes' runs of consecutive positions hits distinct banks.
__host__ __device__ constexpr int sg_pad(int q, int kpt) { return q + q / kpt; }

// Word offset of the reduced-bin arrays (one per digit, 2048 / CL words each) in the
// dynamic shared memory: after the padded score window, rounded up to 4 words
// (uint4 accesses).
__host__ __device__ constexpr int sg_red_offset(int chunk, int radius, int kpt) {
  return (sg_pad(chunk + 2 * radius, kpt) + 1 + 3) & ~3;
}

struct __align__(16) SgShared {  // static part of the shared memory
  uint32_t hist[2048];  // this CTA's histogram of the current digit
  int itmp[33];
  float ftmp[SG_NW];
  float fmax_slot;      // this CTA's largest pooled value (read by the cluster)
  int cnt_slot[2];      // this CTA's (> T, == T) counts (read by the cluster)
  int sel[2];           // selected bin, remaining k
  uint32_t kbig;        // key of the protected tail (amax + 1)
  int ncand;            // keys left after the first digit (candidate list length)
  int before[2];        // keys this CTA writes after (cluster prefix), ties kept here
};

// Cluster barrier split into its two halves: arrive publishes this thread's
// earlier shared-memory writes to the cluster, wait makes the others' visible.
__device__ __forceinline__ void sg_cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void sg_cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// RT: the pooling radius when known at compile time (pooling in registers), or -1.
// KPT: positions per thread (8, 16 or 32).
// One row (srow: its Lk scores) of the selection, run by the calling CTA's whole
// cluster; the kept positions go to orow[0 .. keep_len). `waited`: the caller has
// already waited for the kernel before this one.
template <int RT, int KPT>
__device__ __forceinline__ void sg_select_row(const float* __restrict__ srow, int Lk, int chunk, int radius_rt,
                                              int protect, int keep_len, int64_t* __restrict__ orow0,
                                              bool waited) {
  const int radius = RT >= 0 ? RT : radius_rt;
  cg::cluster_group cluster = cg::this_cluster();
  const int CL = (int)cluster.num_blocks();
  const int r = (int)cluster.block_rank();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  __shared__ SgShared S;
  extern __shared__ uint32_t dyn[];
  float* buf = reinterpret_cast<float*>(dyn);  // padded window of positions [j0 - radius, j1 + radius)
  uint32_t* cand = dyn;                        // candidate keys, once the keys are in registers
  // [3][2048 / CL] reduced bins, read as uint4: 16-byte aligned whatever chunk is
  uint32_t* red = dyn + sg_red_offset(chunk, radius, KPT);
  for (int i = tid; i < 3 * (2048 / CL); i += SG_NT) red[i] = 0;
  if (tid == 0) S.ncand = 0;
  sg_cluster_arrive();  // waited for before the first adds into another CTA's arrays

  const int j0 = min(Lk, r * chunk), j1 = min(Lk, j0 + chunk);
  const int n = j1 - j0;
  if (!waited) pdl_wait();  // the scores come from the kernel before this one
  pdl_launch_dependents();  // the gather may be scheduled on the SMs left free
  const int pstart = Lk - protect;

  // ---- 1. sliding max --------------------------------------------------------
  // window index q <-> row position j0 - radius + q; -inf outside the row, as
  // max_pool1d pads
  const int Q = n + 2 * radius;
  const int jb = j0 - radius;
  for (int q = tid; q < Q; q += 8 * SG_NT) {  // 8 independent loads in flight per thread
    float v8[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int qq = q + u * SG_NT, j = jb + qq;
      v8[u] = (qq < Q && j >= 0 && j < Lk) ? __ldg(srow + j) : -INFINITY;
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int qq = q + u * SG_NT;
      if (qq < Q) buf[sg_pad(qq, KPT)] = v8[u];
    }
  }
  __syncthreads();
  // this thread: chunk positions x0 + u, u < nv
  const int x0 = KPT * tid;
  const int nv = max(0, min(KPT, n - x0));
  float pooled[KPT];
  if (RT >= 0) {
    constexpr int R = RT >= 0 ? RT : 0;
    constexpr int W = 2 * R + 1;
    constexpr int WN = KPT + 2 * R;
    constexpr int P = W >= 16 ? 16 : (W >= 8 ? 8 : (W >= 4 ? 4 : (W >= 2 ? 2 : 1)));
    static_assert(W <= 2 * P, "window covered by two spans");
    float v[WN];
#pragma unroll
    for (int i = 0; i < WN; ++i) {
      const int q = x0 + i;
      v[i] = q < Q ? buf[sg_pad(q, KPT)] : -INFINITY;
    }
    // doubling in place: after the step of span sp, v[i] = max of the inputs [i, i + 2 sp)
#pragma unroll
    for (int sp = 1; sp < P; sp *= 2) {
#pragma unroll
      for (int i = 0; i + sp < WN; ++i) v[i] = fmaxf(v[i], v[i + sp]);
    }
    // [u, u + W) = [u, u + P) U [u + W - P, u + W)
#pragma unroll
    for (int u = 0; u < KPT; ++u) pooled[u] = fmaxf(v[u], v[u + W - P]);
  } else {
#pragma unroll
    for (int u = 0; u < KPT; ++u) {
      float m = -INFINITY;
      for (int i = 0; i <= 2 * radius; ++i) {
        const int q = x0 + u + i;
        if (q < Q) m = fmaxf(m, buf[sg_pad(q, KPT)]);
      }
      pooled[u] = m;
    }
  }
  uint32_t key[KPT];
  float lmax = -INFINITY;
#pragma unroll
  for (int u = 0; u < KPT; ++u) {
    key[u] = ordered_key(pooled[u]);
    if (u < nv) lmax = fmaxf(lmax, pooled[u]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) lmax = fmaxf(lmax, __shfl_xor_sync(0xffffffffu, lmax, o));
  if (lane == 0) S.ftmp[warp] = lmax;
  __syncthreads();
  if (tid == 0) {
    float m = S.ftmp[0];
    for (int w = 1; w < SG_NW; ++w) m = fmaxf(m, S.ftmp[w]);
    S.fmax_slot = m;
  }
  const int ip = pstart - j0 - x0;  // this thread's first protected position (may be <= 0 or >= KPT)

  // ---- 2. radix select over the cluster -------------------------------------
  uint32_t prefix = 0, pmask = 0;
  int k = keep_len;
#pragma unroll 1
  for (int pass = 0; pass < 3; ++pass) {
    const int sh = pass == 0 ? 21 : (pass == 1 ? 10 : 0);
    const int nb = pass == 2 ? 1024 : 2048;
    const uint32_t dmask = (uint32_t)(nb - 1);
    const int per = nb / CL;  // bins per owner; CL is a power of two, so a multiple of 4
    uint32_t* redp = red + pass * (2048 / CL);
    for (int i = tid; i < nb; i += SG_NT) S.hist[i] = 0;
    __syncthreads();
    // Pooled scores form plateaus and share few exponents, so neighbouring
    // positions mostly fall into the same bin: each run of equal bins is added
    // once. The protected tail is left out of the first digit (its key is not
    // known yet); the later digits run over the candidate list, the keys that
    // matched the first digit.
    if (pass == 0) {
      uint32_t cur = 0xffffffffu, run = 0;
#pragma unroll
      for (int u = 0; u < KPT; ++u) {
        const uint32_t b = (u < nv && u < ip) ? (key[u] >> 21) : 0xffffffffu;
        if (b != cur) {
          if (cur != 0xffffffffu) atomicAdd(&S.hist[cur], run);
          cur = b;
          run = 1;
        } else {
          ++run;
        }
      }
      if (cur != 0xffffffffu) atomicAdd(&S.hist[cur], run);
    } else {
      const int ns = S.ncand;
#pragma unroll 4
      for (int base = 0; base < ns; base += SG_NT) {
        const int i = base + tid;
        uint32_t bin = 0xffffffffu;
        if (i < ns) {
          const uint32_t kk = cand[i];
          if ((kk & pmask) == prefix) bin = (kk >> sh) & dmask;
        }
        const uint32_t prev = __shfl_up_sync(0xffffffffu, bin, 1);
        const bool starts = lane == 0 || prev != bin;
        const uint32_t heads = __ballot_sync(0xffffffffu, starts);
        if (starts && bin != 0xffffffffu) {
          const uint32_t after = heads & ~((2u << lane) - 1u);  // run starts past this lane
          const int end = after ? __ffs(after) - 1 : 32;
          atomicAdd(&S.hist[bin], (uint32_t)(end - lane));
        }
      }
    }
    __syncthreads();
    if (pass == 0) sg_cluster_wait();  // every owner has cleared its arrays (arrive at the start)
    for (int bin = tid; bin < nb; bin += SG_NT) {
      const uint32_t c = S.hist[bin];
      if (c) {
        const int owner = bin / per;
        atomicAdd(cluster.map_shared_rank(redp, owner) + (bin - owner * per), c);
      }
    }
    sg_cluster_arrive();  // this CTA's adds (and, before the first digit, its maximum) are done
    sg_cluster_wait();
    if (pass == 0 && warp == 0) {  // row maximum from the CTA maxima; key of the protected tail
      float m = lane < CL ? *cluster.map_shared_rank(&S.fmax_slot, lane) : -INFINITY;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      if (lane == 0) S.kbig = ordered_key(m + 1.0f);
    }
    // every CTA reads all reduced bins (thread t: bins [4t, 4t + 4)) and finds the
    // bin holding the k-th largest key
    int cnt[4] = {0, 0, 0, 0};
    if (tid * 4 < nb) {
      const int b = tid * 4, owner = b / per;
      const uint4 c4 = *reinterpret_cast<const uint4*>(cluster.map_shared_rank(redp, owner) + (b - owner * per));
      cnt[0] = (int)c4.x;
      cnt[1] = (int)c4.y;
      cnt[2] = (int)c4.z;
      cnt[3] = (int)c4.w;
    }
    if (pass == 0) {
      __syncthreads();
      if (protect > 0) {  // the whole protected tail shares one key
        const int bb = (int)((S.kbig >> sh) & dmask) - tid * 4;
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (bb == u) cnt[u] += protect;
      }
    }
    const int my_sum = cnt[0] + cnt[1] + cnt[2] + cnt[3];
    int total;
    const int below = sg_block_excl_scan(my_sum, S.itmp, &total);
    int above = total - below - my_sum;  // keys in higher bins
#pragma unroll
    for (int u = 3; u >= 0; --u) {
      if (above < k && k <= above + cnt[u]) {
        S.sel[0] = tid * 4 + u;
        S.sel[1] = k - above;
      }
      above += cnt[u];
    }
    __syncthreads();
    prefix |= ((uint32_t)S.sel[0]) << sh;
    pmask |= dmask << sh;
    k = S.sel[1];
    if (pass == 0) {
      // protected positions carry the key of amax + 1 from here on; the keys that
      // match the first digit go to the candidate list (in any order: the later
      // digits only count them)
      const uint32_t kbig = S.kbig;
      int c = 0;
#pragma unroll
      for (int u = 0; u < KPT; ++u) {
        if (u >= ip) key[u] = kbig;
        c += (u < nv && (key[u] & pmask) == prefix) ? 1 : 0;
      }
      int inc = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += t;
      }
      int base = 0;
      if (lane == 31 && inc > 0) base = atomicAdd(&S.ncand, inc);
      int pos = __shfl_sync(0xffffffffu, base, 31) + inc - c;
#pragma unroll
      for (int u = 0; u < KPT; ++u)
        if (u < nv && (key[u] & pmask) == prefix) cand[pos++] = key[u];
    }
    __syncthreads();
  }
  const uint32_t T = prefix;
  const int need_eq = k;

  // ---- 3. ordered compaction -------------------------------------------------
  // Kept: every key > T and the first need_eq keys == T in position order (ties to
  // the lower index). Threads own consecutive positions, so one block scan of the
  // packed (> T, == T) counts ranks every position of the CTA.
  int cgt = 0, ceq = 0;
#pragma unroll
  for (int u = 0; u < KPT; ++u) {
    if (u < nv) {
      cgt += key[u] > T ? 1 : 0;
      ceq += key[u] == T ? 1 : 0;
    }
  }
  int ctot;
  const int cpre = sg_block_excl_scan(cgt | (ceq << 16), S.itmp, &ctot);  // counts < 2^16
  if (tid == 0) {
    S.cnt_slot[0] = ctot & 0xffff;
    S.cnt_slot[1] = ctot >> 16;
  }
  sg_cluster_arrive();
  sg_cluster_wait();
  if (warp == 0) {
    // CTAs c < r come first: all their keys > T, and the first (need_eq - ties
    // before c) of their ties
    int g = 0, e = 0;
    if (lane < r) {
      const int* sl = cluster.map_shared_rank(S.cnt_slot, lane);
      g = sl[0];
      e = sl[1];
    }
    int einc = e;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, einc, o);
      if (lane >= o) einc += t;
    }
    int term = (lane < r) ? g + max(0, min(e, need_eq - (einc - e))) : 0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) term += __shfl_xor_sync(0xffffffffu, term, o);
    const int eq_all = __shfl_sync(0xffffffffu, einc, 31);
    if (lane == 0) {
      S.before[0] = term;
      S.before[1] = eq_all;
    }
  }
  __syncthreads();
  const int out_before = S.before[0], eq_before = S.before[1];
  const int need_local = max(0, need_eq - eq_before);  // ties this CTA keeps, lowest index first
  int64_t* orow = orow0 + out_before;
  int g = cpre & 0xffff, e = cpre >> 16;
  const int jx = j0 + x0;
#pragma unroll
  for (int u = 0; u < KPT; ++u) {
    if (u < nv) {
      const bool gt = key[u] > T, eq = key[u] == T;
      if (gt || (eq && e < need_local)) {
        const int pos = g + min(e, need_local);
        if (out_before + pos < keep_len) orow[pos] = jx + u;
      }
      g += gt ? 1 : 0;
      e += eq ? 1 : 0;
    }
  }
  cluster.sync();  // keep this CTA's shared memory alive until the cluster has read it
}

// Rows of one length: row blockIdx.x / CL of scores [rows, Lk] into keep_idx [rows, keep_len].
template <int RT, int KPT>
__global__ void __launch_bounds__(SG_NT, 1) cluster_select_kernel(const float* __restrict__ scores, int Lk,
                                                                  int chunk, int radius_rt, int protect,
                                                                  int keep_len, int64_t* __restrict__ keep_idx) {
  const int row = blockIdx.x / (int)cg::this_cluster().num_blocks();
  sg_select_row<RT, KPT>(scores + (size_t)row * Lk, Lk, chunk, radius_rt, protect, keep_len,
                         keep_idx + (size_t)row * keep_len, false);
}

// A ragged batch: row blockIdx.x / CL of the batch belongs to the sequence the table
// names; its length, chunk and keep_len (the keep_len rule, evaluated here) are the
// sequence's own. The dynamic shared memory is sized for the longest row.
template <int RT, int KPT>
__global__ void __launch_bounds__(SG_NT, KPT <= 16 ? 2 : 1) cluster_select_varlen_kernel(const __grid_constant__ VarlenTable t,
                                                                         int radius_rt) {
  cg::cluster_group cluster = cg::this_cluster();
  const int CL = (int)cluster.num_blocks();
  const int row = blockIdx.x / CL;
  const int s = varlen_seq_of(t, row);
  const VarlenSeq& q = t.s[s];
  pdl_wait();  // the scores (and possibly total_tokens / max_keep_len) come from earlier kernels
  const int keep_len = varlen_keep_len(t, s);
  if (row == q.row0 && cluster.block_rank() == 0 && threadIdx.x == 0) t.keep_len_out[s] = keep_len;
  if (keep_len == 0) return;  // the whole cluster returns here, before any cluster barrier
  const int lk = q.lk, b = row - q.row0;
  sg_select_row<RT, KPT>(t.scores + q.score_off + (size_t)b * lk, lk, (lk + CL - 1) / CL, radius_rt,
                         min(t.protect, lk), keep_len, q.keep_idx + (size_t)b * q.cap, true);
}

}  // namespace

// Cluster size and chunk for a row of Lk positions; 0 if the row does not fit.
// The largest cluster considered gives each CTA <= 4096 positions (up to 16 CTAs);
// a cluster of half that size is the other candidate (see launch_cluster_select).
static int sg_kpt(int chunk) { return chunk <= 8 * SG_NT ? 8 : (chunk <= 16 * SG_NT ? 16 : 32); }

static int sg_chunk(int Lk, int radius, int cl, int* chunk_out, size_t* smem_out) {
  const int chunk = (Lk + cl - 1) / cl;
  if (chunk > 32 * SG_NT) return 0;
  const size_t smem = ((size_t)sg_red_offset(chunk, radius, sg_kpt(chunk)) + 3 * (2048 / cl)) * 4;
  if (smem + sizeof(SgShared) > 227 * 1024) return 0;
  *chunk_out = chunk;
  *smem_out = smem;
  return cl;
}

static int sg_cluster_for(int Lk, int radius, int* chunk_out, size_t* smem_out) {
  int cl = 1;
  while (cl < SG_MAXCL && (Lk + cl - 1) / cl > 4096) cl *= 2;
  return sg_chunk(Lk, radius, cl, chunk_out, smem_out);
}

bool select_gather_supported(int Lk, int kernel_size) {
  int chunk;
  size_t smem;
  return sg_cluster_for(Lk, kernel_size / 2, &chunk, &smem) > 0;
}

using SgKernel = void (*)(const float*, int, int, int, int, int, int64_t*);
using SgKernelV = void (*)(VarlenTable, int);
constexpr int SG_VARIANTS = 6;

// kernel for the radius (5: the default kernel_size 11) and positions per thread
static int sg_variant(bool r5, int kpt) { return (r5 ? 3 : 0) + (kpt == 8 ? 0 : (kpt == 16 ? 1 : 2)); }

static SgKernel sg_kernel(bool r5, int kpt, int* variant) {
  static const SgKernel table[SG_VARIANTS] = {
      cluster_select_kernel<-1, 8>, cluster_select_kernel<-1, 16>, cluster_select_kernel<-1, 32>,
      cluster_select_kernel<5, 8>,  cluster_select_kernel<5, 16>,  cluster_select_kernel<5, 32>};
  *variant = sg_variant(r5, kpt);
  return table[*variant];
}

static SgKernelV sg_kernel_varlen(int variant) {
  static const SgKernelV table[SG_VARIANTS] = {
      cluster_select_varlen_kernel<-1, 8>, cluster_select_varlen_kernel<-1, 16>,
      cluster_select_varlen_kernel<-1, 32>, cluster_select_varlen_kernel<5, 8>,
      cluster_select_varlen_kernel<5, 16>, cluster_select_varlen_kernel<5, 32>};
  return table[variant];
}

// Function attributes, set once per device and kernel: the largest dynamic
// shared memory any chunk can ask for, and 16-CTA clusters.
template <typename K>
static int sg_prepare_kernel(K kern, DeviceOnce& done, size_t smem) {
  const int max_dyn = 227 * 1024 - (int)sizeof(SgShared);
  if (smem > (size_t)max_dyn) return fail(DROPKV_ERR_UNSUPPORTED, "cluster select needs %zu bytes", smem);
  int dev = 0;
  cudaGetDevice(&dev);
  if (done.done(dev)) return DROPKV_OK;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, max_dyn) != cudaSuccess)
    return fail(DROPKV_ERR_CUDA, "cannot set shared memory size %d for the cluster select", max_dyn);
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)
    return fail(DROPKV_ERR_CUDA, "cannot allow 16-CTA clusters for the cluster select");
  done.mark(dev);
  return DROPKV_OK;
}

static int sg_prepare(SgKernel kern, int variant, size_t smem) {
  static DeviceOnce done[SG_VARIANTS];
  return sg_prepare_kernel(kern, done[variant], smem);
}

static int sg_prepare_varlen(int variant, size_t smem) {
  static DeviceOnce done[SG_VARIANTS];
  return sg_prepare_kernel(sg_kernel_varlen(variant), done[variant], smem);
}

// Clusters of `cl` CTAs that can be resident at once on this device (a cluster
// must fit in one GPC, and GPCs differ in size), cached per device, variant,
// cluster size and 8 KB step of dynamic shared memory (the query uses the step's
// upper end, so the answer is never too high).
static int sg_active_clusters(SgKernel kern, int variant, int cl, size_t smem) {
  constexpr int kDevs = 16, kSteps = 29;  // 29 steps of 8 KB cover 227 KB
  static std::atomic<int> cache[SG_VARIANTS][5][kDevs][kSteps];  // zero: not queried yet
  int dev = 0;
  cudaGetDevice(&dev);
  int lg = 0;
  while ((1 << lg) < cl) ++lg;
  const int step = (int)std::min<size_t>(kSteps - 1, smem / 8192);
  const size_t smem_q = std::min<size_t>((size_t)(step + 1) * 8192, 227 * 1024 - sizeof(SgShared));  // <= max_dyn
  if (dev >= 0 && dev < kDevs) {
    const int c = cache[variant][lg][dev][step].load(std::memory_order_relaxed);
    if (c > 0) return c;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(cl);
  cfg.blockDim = dim3(SG_NT);
  cfg.dynamicSmemBytes = std::max(smem, smem_q);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cl;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n < 1) {
    cudaGetLastError();  // clear the query's error; assume every cluster is resident
    return 1 << 20;
  }
  if (dev >= 0 && dev < kDevs) cache[variant][lg][dev][step].store(n, std::memory_order_relaxed);
  return n;
}

struct SgChoice {
  int cl, chunk, variant;
  size_t smem;
};

// Cluster size, chunk and kernel variant for BH rows of (at most) Lk positions.
static int plan_cluster_select(int BH, int Lk, int kernel_size, SgChoice* out) {
  const int radius = kernel_size / 2;
  const bool r5 = radius == 5;
  int chunk;
  size_t smem;
  int cl = sg_cluster_for(Lk, radius, &chunk, &smem);
  if (!cl) return fail(DROPKV_ERR_UNSUPPORTED, "row of %d positions too long for the cluster select", Lk);
  int variant;
  SgKernel kern = sg_kernel(r5, sg_kpt(chunk), &variant);
  int rc = sg_prepare(kern, variant, smem);
  if (rc) return rc;
  // Rows run one cluster each; rows beyond the resident clusters wait for another
  // wave. Estimated time per wave: a fixed ~6 us of barriers plus ~0.9 us per
  // position of a thread (measured on B200). Smaller clusters (more positions per
  // thread) are considered only while the rows need more than one wave.
  auto cost = [&](SgKernel kr, int var, int c, int ch, size_t sm, int* waves_out) {
    const int act = sg_active_clusters(kr, var, c, sm);
    *waves_out = (BH + act - 1) / act;
    return *waves_out * (6.0 + 0.9 * ch / (double)SG_NT);
  };
  int waves;
  double best = cost(kern, variant, cl, chunk, smem, &waves);
  for (int c = cl / 2; c >= 1 && waves > 1; c /= 2) {
    int ch;
    size_t sm;
    if (!sg_chunk(Lk, radius, c, &ch, &sm)) break;  // chunks only grow from here
    int var;
    SgKernel kr = sg_kernel(r5, sg_kpt(ch), &var);
    if ((rc = sg_prepare(kr, var, sm))) return rc;
    int w;
    const double t = cost(kr, var, c, ch, sm, &w);
    if (t < best) {
      best = t;
      cl = c;
      chunk = ch;
      smem = sm;
      variant = var;
    }
    waves = w;
  }
  out->cl = cl;
  out->chunk = chunk;
  out->variant = variant;
  out->smem = smem;
  return DROPKV_OK;
}

// cluster launch of `rows` rows of `cl` CTAs, allowed to start while the kernel
// before it finishes (programmatic dependent launch)
template <typename K, typename... Args>
static int sg_launch(K kern, int rows, const SgChoice& c, cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(rows * c.cl);
  cfg.blockDim = dim3(SG_NT);
  cfg.dynamicSmemBytes = c.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = c.cl;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, args...);
  if (e != cudaSuccess) return fail(DROPKV_ERR_CUDA, "cluster select launch: %s", cudaGetErrorString(e));
  return check_launch("cluster_select");
}

static int launch_cluster_select(const float* scores, int BH, int Lk, int kernel_size, int protect, int keep_len,
                                 int64_t* keep_idx, cudaStream_t st) {
  SgChoice c;
  int rc = plan_cluster_select(BH, Lk, kernel_size, &c);
  if (rc) return rc;
  int variant;
  SgKernel kern = sg_kernel(kernel_size / 2 == 5, sg_kpt(c.chunk), &variant);
  return sg_launch(kern, BH, c, st, scores, Lk, c.chunk, kernel_size / 2, protect, keep_len, keep_idx);
}

// Selection into keep_idx and, when K/V are given, the gather of the kept rows.
int launch_select_gather(const float* scores, int BH, int Lk, int kernel_size, int protect, int keep_len,
                         int64_t* keep_idx, const void* k, const void* v, int elem_bytes, int D, void* ko,
                         void* vo, cudaStream_t st, int64_t in_sh, int64_t out_sh, int Hkv, int64_t in_sb,
                         int64_t in_ss) {
  int rc = launch_cluster_select(scores, BH, Lk, kernel_size, protect, keep_len, keep_idx, st);
  if (rc || k == nullptr) return rc;
  return launch_gather(k, v, elem_bytes, BH, Lk, D, keep_idx, keep_len, ko, vo, st, in_sh, out_sh, Hkv, in_sb, in_ss);
}

int launch_gather_varlen(const VarlenTable& t, int elem_bytes, int D, cudaStream_t st);

// A ragged batch: the plan of the longest row serves every row (a shorter row's
// chunk is smaller, so the same shared memory holds it).
int launch_select_gather_varlen(const VarlenTable& t, int kernel_size, int elem_bytes, int D, cudaStream_t st) {
  if (t.rows < 1) return DROPKV_OK;
  int lk_max = 1;
  for (int i = 0; i < t.n; ++i) lk_max = std::max(lk_max, t.s[i].lk);
  SgChoice c;
  int rc = plan_cluster_select(t.rows, lk_max, kernel_size, &c);
  if (rc) return rc;
  if ((rc = sg_prepare_varlen(c.variant, c.smem))) return rc;
  if ((rc = sg_launch(sg_kernel_varlen(c.variant), t.rows, c, st, t, kernel_size / 2))) return rc;
  return launch_gather_varlen(t, elem_bytes, D, st);
}

}  // namespace dropkv
