// Compaction of the kept K/V rows: k_out[bh, i, :] = k[bh, keep_idx[bh, i], :]
// (and the same for V), a bit-exact copy.  Replaces dropkv_cache.py:479-491
// (torch.gather along the sequence axis with the index expanded over D).
//
// Each thread moves one VW-byte chunk of one row of K and of V; consecutive
// threads cover consecutive chunks of a row, so every warp reads and writes whole
// 128-byte lines.  Indices outside [0, Lk) produce zero rows (no trap).
#include <algorithm>

#include "common.cuh"

namespace dropkv {
namespace {

// in_sh / out_sh: vectors between consecutive heads of the input and the output.
template <typename VT>
__global__ void __launch_bounds__(256) gather_kernel(const VT* __restrict__ k, const VT* __restrict__ v,
                                                     const int64_t* __restrict__ idx, int Lk, int keep_len,
                                                     int CR, VT* __restrict__ ko, VT* __restrict__ vo,
                                                     int64_t in_sh, int64_t out_sh) {
  const int bh = blockIdx.y;
  const int64_t n = (int64_t)keep_len * CR;
  const int64_t* ib = idx + (size_t)bh * keep_len;
  const VT* kb = k + (size_t)bh * in_sh;
  const VT* vb = v + (size_t)bh * in_sh;
  VT* kob = ko + (size_t)bh * out_sh;
  VT* vob = vo + (size_t)bh * out_sh;
  for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < n;
       c += (int64_t)gridDim.x * blockDim.x) {
    int64_t i = c / CR;
    int col = (int)(c - i * CR);
    int64_t src = ib[i];
    VT a, b;
    if (src >= 0 && src < Lk) {
      a = kb[src * CR + col];
      b = vb[src * CR + col];
    } else {
      a = VT{};
      b = VT{};
    }
    kob[i * CR + col] = a;
    vob[i * CR + col] = b;
  }
}

template <typename VT>
int launch_vec(const void* k, const void* v, int BH, int Lk, int row_bytes, const int64_t* idx,
               int keep_len, void* ko, void* vo, cudaStream_t st, int64_t in_sh_bytes, int64_t out_sh_bytes) {
  int CR = row_bytes / (int)sizeof(VT);
  int64_t n = (int64_t)keep_len * CR;
  int bx = (int)std::min<int64_t>((n + 255) / 256, 4096);
  if (bx < 1) bx = 1;
  dim3 grid(bx, BH);
  gather_kernel<VT><<<grid, 256, 0, st>>>(reinterpret_cast<const VT*>(k), reinterpret_cast<const VT*>(v),
                                          idx, Lk, keep_len, CR, reinterpret_cast<VT*>(ko),
                                          reinterpret_cast<VT*>(vo), in_sh_bytes / (int64_t)sizeof(VT),
                                          out_sh_bytes / (int64_t)sizeof(VT));
  return check_launch("gather");
}

bool aligned(const void* p, int a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

}  // namespace

int launch_gather(const void* k, const void* v, int elem_bytes, int BH, int Lk, int D,
                  const int64_t* keep_idx, int keep_len, void* k_out, void* v_out, cudaStream_t st,
                  int64_t in_sh, int64_t out_sh) {
  if (keep_len == 0 || BH == 0) return DROPKV_OK;
  const int row_bytes = D * elem_bytes;
  const int64_t in_b = (in_sh ? in_sh : (int64_t)Lk * D) * elem_bytes;
  const int64_t out_b = (out_sh ? out_sh : (int64_t)keep_len * D) * elem_bytes;
  for (int w : {16, 8, 4, 2}) {
    if (row_bytes % w == 0 && in_b % w == 0 && out_b % w == 0 && aligned(k, w) && aligned(v, w) &&
        aligned(k_out, w) && aligned(v_out, w)) {
      switch (w) {
        case 16: return launch_vec<uint4>(k, v, BH, Lk, row_bytes, keep_idx, keep_len, k_out, v_out, st, in_b, out_b);
        case 8: return launch_vec<uint2>(k, v, BH, Lk, row_bytes, keep_idx, keep_len, k_out, v_out, st, in_b, out_b);
        case 4: return launch_vec<uint32_t>(k, v, BH, Lk, row_bytes, keep_idx, keep_len, k_out, v_out, st, in_b, out_b);
        case 2: return launch_vec<uint16_t>(k, v, BH, Lk, row_bytes, keep_idx, keep_len, k_out, v_out, st, in_b, out_b);
      }
    }
  }
  return fail(DROPKV_ERR_ARG, "gather: K/V and outputs must be at least 2-byte aligned");
}

}  // namespace dropkv
