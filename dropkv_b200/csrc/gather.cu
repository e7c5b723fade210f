// Compaction of the kept K/V rows: k_out[bh, i, :] = k[bh, keep_idx[bh, i], :]
// (and the same for V), a bit-exact copy.  Replaces dropkv_cache.py:479-491
// (torch.gather along the sequence axis with the index expanded over D).
//
// Each thread moves VW-byte chunks of rows of K and of V; consecutive threads
// cover consecutive chunks of a row, so every warp reads and writes whole
// 128-byte lines.  Indices outside [0, Lk) produce zero rows (no trap).
#include <algorithm>

#include "common.cuh"

namespace dropkv {
namespace {

constexpr int GT_NT = 256;  // threads per block
constexpr int GT_U = 2;     // chunks per thread and step: 2 K and 2 V loads in flight

// One row: ko[i, :] = kb[ib[i], :] and vo[i, :] = vb[ib[i], :] for i < keep_len, rows
// of CR vectors, input rows RS vectors apart. Block x of the row handles steps x,
// x + gridDim.x, ...; a step is GT_U * GT_NT consecutive chunks, and all its index
// and data loads are issued before its stores.
template <typename VT>
__device__ __forceinline__ void gather_row(const VT* __restrict__ kb, const VT* __restrict__ vb,
                                           const int64_t* __restrict__ ib, int Lk, int keep_len, int CR,
                                           VT* __restrict__ kob, VT* __restrict__ vob, int64_t RS) {
  const int64_t n = (int64_t)keep_len * CR;
  for (int64_t c0 = (int64_t)blockIdx.x * (GT_U * GT_NT) + threadIdx.x; c0 < n;
       c0 += (int64_t)gridDim.x * (GT_U * GT_NT)) {
    int64_t src[GT_U], i[GT_U];
    int col[GT_U];
#pragma unroll
    for (int u = 0; u < GT_U; ++u) {
      const int64_t c = c0 + u * GT_NT;
      i[u] = c / CR;
      col[u] = (int)(c - i[u] * CR);
      src[u] = c < n ? ib[i[u]] : -1;
    }
    VT a[GT_U], b[GT_U];
#pragma unroll
    for (int u = 0; u < GT_U; ++u) {
      if (src[u] >= 0 && src[u] < Lk) {
        a[u] = kb[src[u] * RS + col[u]];
        b[u] = vb[src[u] * RS + col[u]];
      } else {
        a[u] = VT{};
        b[u] = VT{};
      }
    }
#pragma unroll
    for (int u = 0; u < GT_U; ++u) {
      if (c0 + u * GT_NT < n) {
        kob[i[u] * CR + col[u]] = a[u];
        vob[i[u] * CR + col[u]] = b[u];
      }
    }
  }
}

// Row bh = b * Hkv + h; in_sb / in_sh / in_rs: vectors between consecutive
// sequences, heads and keys of the input; out_sh: between consecutive rows of the
// output.
template <typename VT>
__global__ void __launch_bounds__(GT_NT) gather_kernel(const VT* __restrict__ k, const VT* __restrict__ v,
                                                       const int64_t* __restrict__ idx, int Lk, int keep_len,
                                                       int CR, VT* __restrict__ ko, VT* __restrict__ vo, int Hkv,
                                                       int64_t in_sb, int64_t in_sh, int64_t in_rs,
                                                       int64_t out_sh) {
  const int bh = blockIdx.y;
  const int64_t in_off = (int64_t)(bh / Hkv) * in_sb + (int64_t)(bh % Hkv) * in_sh;
  pdl_wait();  // keep_idx may come from the kernel before this one
  gather_row<VT>(k + in_off, v + in_off, idx + (size_t)bh * keep_len, Lk, keep_len, CR, ko + (size_t)bh * out_sh,
                 vo + (size_t)bh * out_sh, in_rs);
}

// A ragged batch: row blockIdx.y of the table's batch, with its sequence's
// lengths; keep_len is the one the selection wrote to t.keep_len_out.
template <typename VT>
__global__ void __launch_bounds__(GT_NT) gather_varlen_kernel(const __grid_constant__ VarlenTable t, int CR) {
  const int row = blockIdx.y;
  const int s = varlen_seq_of(t, row);
  const VarlenSeq& q = t.s[s];
  const int b = row - q.row0;
  pdl_wait();  // keep_idx and keep_len_out come from the selection
  const int keep_len = t.keep_len_out[s];
  const int64_t in_sh = (int64_t)q.lk * CR, out_sh = (int64_t)q.cap * CR;
  gather_row<VT>(reinterpret_cast<const VT*>(q.k) + b * in_sh, reinterpret_cast<const VT*>(q.v) + b * in_sh,
                 q.keep_idx + (size_t)b * q.cap, q.lk, keep_len, CR, reinterpret_cast<VT*>(q.k_out) + b * out_sh,
                 reinterpret_cast<VT*>(q.v_out) + b * out_sh, CR);
}

template <typename VT>
int launch_vec(const void* k, const void* v, int BH, int Lk, int row_bytes, const int64_t* idx,
               int keep_len, void* ko, void* vo, cudaStream_t st, int64_t in_sh_bytes, int64_t out_sh_bytes,
               int Hkv, int64_t in_sb_bytes, int64_t in_rs_bytes) {
  int CR = row_bytes / (int)sizeof(VT);
  int64_t n = (int64_t)keep_len * CR;
  // one wave of blocks over the GPU (8 per SM), with the steps of a row spread
  // evenly over its blocks
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t steps = (n + GT_U * GT_NT - 1) / (GT_U * GT_NT);
  const int64_t target = std::max<int64_t>(1, (int64_t)sms * (2048 / GT_NT) / BH);
  const int64_t per_block = (steps + target - 1) / target;
  int bx = (int)std::min<int64_t>((steps + per_block - 1) / per_block, 65535);
  if (bx < 1) bx = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(bx, BH);
  cfg.blockDim = dim3(GT_NT);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // may start as the selection ends
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, gather_kernel<VT>, reinterpret_cast<const VT*>(k),
                                     reinterpret_cast<const VT*>(v), idx, Lk, keep_len, CR,
                                     reinterpret_cast<VT*>(ko), reinterpret_cast<VT*>(vo), Hkv,
                                     in_sb_bytes / (int64_t)sizeof(VT), in_sh_bytes / (int64_t)sizeof(VT),
                                     in_rs_bytes / (int64_t)sizeof(VT), out_sh_bytes / (int64_t)sizeof(VT));
  if (e != cudaSuccess) return fail(DROPKV_ERR_CUDA, "gather launch: %s", cudaGetErrorString(e));
  return check_launch("gather");
}

bool aligned(const void* p, int a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

template <typename VT>
int launch_varlen_vec(const VarlenTable& t, int row_bytes, cudaStream_t st) {
  const int CR = row_bytes / (int)sizeof(VT);
  int cap_max = 1;
  for (int i = 0; i < t.n; ++i) cap_max = std::max(cap_max, t.s[i].cap);
  const int64_t n = (int64_t)cap_max * CR;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t steps = (n + GT_U * GT_NT - 1) / (GT_U * GT_NT);
  const int64_t target = std::max<int64_t>(1, (int64_t)sms * (2048 / GT_NT) / t.rows);
  const int64_t per_block = (steps + target - 1) / target;
  int bx = (int)std::min<int64_t>((steps + per_block - 1) / per_block, 65535);
  if (bx < 1) bx = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(bx, t.rows);
  cfg.blockDim = dim3(GT_NT);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, gather_varlen_kernel<VT>, t, CR);
  if (e != cudaSuccess) return fail(DROPKV_ERR_CUDA, "varlen gather launch: %s", cudaGetErrorString(e));
  return check_launch("gather_varlen");
}

}  // namespace

int launch_gather(const void* k, const void* v, int elem_bytes, int BH, int Lk, int D,
                  const int64_t* keep_idx, int keep_len, void* k_out, void* v_out, cudaStream_t st,
                  int64_t in_sh, int64_t out_sh, int Hkv, int64_t in_sb, int64_t in_ss) {
  if (keep_len == 0 || BH == 0) return DROPKV_OK;
  const int row_bytes = D * elem_bytes;
  const int64_t sh = in_sh ? in_sh : (int64_t)Lk * D;
  const int64_t in_b = sh * elem_bytes;
  const int64_t sb_b = (in_sb ? in_sb : (int64_t)Hkv * sh) * elem_bytes;
  const int64_t rs_b = (in_ss ? in_ss : (int64_t)D) * elem_bytes;
  const int64_t out_b = (out_sh ? out_sh : (int64_t)keep_len * D) * elem_bytes;
  for (int w : {16, 8, 4, 2}) {
    if (row_bytes % w == 0 && in_b % w == 0 && sb_b % w == 0 && rs_b % w == 0 && out_b % w == 0 && aligned(k, w) &&
        aligned(v, w) && aligned(k_out, w) && aligned(v_out, w)) {
      switch (w) {
        case 16:
          return launch_vec<uint4>(k, v, BH, Lk, row_bytes, keep_idx, keep_len, k_out, v_out, st, in_b, out_b, Hkv,
                                   sb_b, rs_b);
        case 8:
          return launch_vec<uint2>(k, v, BH, Lk, row_bytes, keep_idx, keep_len, k_out, v_out, st, in_b, out_b, Hkv,
                                   sb_b, rs_b);
        case 4:
          return launch_vec<uint32_t>(k, v, BH, Lk, row_bytes, keep_idx, keep_len, k_out, v_out, st, in_b, out_b,
                                      Hkv, sb_b, rs_b);
        case 2:
          return launch_vec<uint16_t>(k, v, BH, Lk, row_bytes, keep_idx, keep_len, k_out, v_out, st, in_b, out_b,
                                      Hkv, sb_b, rs_b);
      }
    }
  }
  return fail(DROPKV_ERR_ARG, "gather: K/V and outputs must be at least 2-byte aligned");
}

// Vector width: the widest that every sequence's rows, pointers and row strides allow.
int launch_gather_varlen(const VarlenTable& t, int elem_bytes, int D, cudaStream_t st) {
  if (t.rows < 1) return DROPKV_OK;
  const int row_bytes = D * elem_bytes;
  for (int w : {16, 8, 4, 2}) {
    bool ok = row_bytes % w == 0;
    for (int i = 0; i < t.n && ok; ++i) {
      const VarlenSeq& q = t.s[i];
      ok = aligned(q.k, w) && aligned(q.v, w) && aligned(q.k_out, w) && aligned(q.v_out, w);
    }
    if (!ok) continue;
    switch (w) {
      case 16: return launch_varlen_vec<uint4>(t, row_bytes, st);
      case 8: return launch_varlen_vec<uint2>(t, row_bytes, st);
      case 4: return launch_varlen_vec<uint32_t>(t, row_bytes, st);
      case 2: return launch_varlen_vec<uint16_t>(t, row_bytes, st);
    }
  }
  return fail(DROPKV_ERR_ARG, "varlen gather: K/V and outputs must be at least 2-byte aligned");
}

}  // namespace dropkv
