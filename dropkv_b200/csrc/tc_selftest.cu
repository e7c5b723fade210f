// Hardware self-test of the tcgen05 / TMA building blocks used by the fused
// scorer: one 128-row tile through each MMA form the scorer issues, compared by
// the caller against a plain matrix product.
//
//   mode 0 (logits form):  out[128][n] = A[128][128] . B[n][128]^T
//                          A by TMA (K-major), B written by threads (K-major)
//   mode 1 (P.V form):     out[128][n] = A[128 keys][128]^T . B[n][128 keys]^T
//                          A by TMA read as an MN-major operand
//   mode 2 / 3:            modes 0 / 1 with 64-wide rows (D = 64)
//   mode 4:                mode 1 with B stored MN-major: rows = keys, n elements
//                          per row under the 2n-byte swizzle (n = 16, 32, 64)
//   mode 5:                mode 4 with N = n split into two swizzle atoms of n/2
//                          columns, the second atom 128 rows further (LBO)
//                          (n = 32, 64, 128)
#include "tc_common.cuh"

namespace dropkv {
namespace {

template <int D>
__global__ void __launch_bounds__(128, 1)
    selftest_kernel(const __grid_constant__ CUtensorMap amap, const uint16_t* __restrict__ b, int n,
                    int pv_form, int mn_major, float* __restrict__ out, int* __restrict__ status) {
  extern __shared__ uint8_t raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
  constexpr int A_BYTES = 128 * D * 2;
  uint8_t* As = sm;
  uint8_t* Bs = sm + A_BYTES;               // regions of n rows x 128 B
  const int b_regions = pv_form ? 2 : D / 64;
  uint64_t* bars = reinterpret_cast<uint64_t*>(Bs + b_regions * n * 128);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 2);
  const int tid = threadIdx.x, warp = tid >> 5;

  if (tid == 0) {
    tc::mbar_init(&bars[0], 1);
    tc::mbar_init(&bars[1], 1);
    tc::fence_mbar_init();
  }
  if (warp == 0) {
    tc::tmem_alloc(tslot, 128);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tslot;

  if (tid == 0) {
    tc::mbar_arrive_expect_tx(&bars[0], A_BYTES);
    for (int r = 0; r < D / 64; ++r)
      tc::tma_load_3d(As + r * 16384, &amap, &bars[0], 64 * r, 0, 0, tc::policy_evict_first());
  }
  // B rows: K-major SW128, 64 elements per region row (mn_major: rows = keys)
  const int bk = pv_form ? 128 : D;  // K extent of B
  for (int i = tid; i < n * bk; i += 128) {
    int row = i / bk, k = i % bk;
    if (mn_major == 2) {  // two atoms of n/2 columns, the second at 128 rows x n bytes
      const int at = n / 2, t = row / at, c = row % at;
      const uint32_t off = (uint32_t)t * 128u * (uint32_t)n +
                           (at == 16 ? tc::swz_offset<32>(k, c)
                                     : (at == 32 ? tc::swz_offset<64>(k, c) : tc::swz_offset<128>(k, c)));
      *reinterpret_cast<uint16_t*>(Bs + off) = b[(size_t)row * bk + k];
    } else if (mn_major) {
      const uint32_t off = n == 16 ? tc::swz_offset<32>(k, row)
                                   : (n == 32 ? tc::swz_offset<64>(k, row) : tc::swz_offset<128>(k, row));
      *reinterpret_cast<uint16_t*>(Bs + off) = b[(size_t)row * bk + k];
    } else {
      uint8_t* reg = Bs + (k / 64) * n * 128;
      *reinterpret_cast<uint16_t*>(reg + tc::sw128_offset(row, k % 64)) = b[(size_t)row * bk + k];
    }
  }
  tc::fence_proxy_async_smem();
  __syncthreads();

  bool ok = true;
  if (tid == 0) {
    ok = tc::mbar_wait(&bars[0], 0, 2000000000ull);
    if (ok) {
      tc::tc_fence_after();
      const uint32_t a0 = tc::smem_addr(As), b0 = tc::smem_addr(Bs);
      if (!pv_form) {
        const uint32_t idesc = tc::idesc_f16(true, 128, n, false, false);
        for (int kk = 0; kk < D / 16; ++kk) {
          uint64_t ad = tc::smem_desc(a0 + (kk / 4) * 16384 + (kk % 4) * 32, 16, 1024);
          uint64_t bd = tc::smem_desc(b0 + (kk / 4) * n * 128 + (kk % 4) * 32, 16, 1024);
          tc::mma_f16(tmem, ad, bd, idesc, kk > 0);
        }
      } else if (!mn_major) {
        const uint32_t idesc = tc::idesc_f16(true, 128, n, true, false);
        const uint32_t lbo = (D == 128) ? 16384 : 0;  // second 64-wide slab (D=64: repeat the first)
        for (int kk = 0; kk < 8; ++kk) {
          uint64_t ad = tc::smem_desc(a0 + kk * 2048, lbo, 1024);
          uint64_t bd = tc::smem_desc(b0 + (kk / 4) * n * 128 + (kk % 4) * 32, 16, 1024);
          tc::mma_f16(tmem, ad, bd, idesc, kk > 0);
        }
      } else if (mn_major == 2) {
        const uint32_t idesc = tc::idesc_f16(true, 128, n, true, true);
        const uint32_t rb = n;  // bytes per key row of one atom (n/2 columns)
        for (int kk = 0; kk < 8; ++kk) {
          uint64_t ad = tc::smem_desc(a0 + kk * 2048, 16384, 1024);
          uint64_t bd = tc::smem_desc(b0 + kk * 16 * rb, 128 * rb, 8 * rb, tc::layout_for_row_bytes(rb));
          tc::mma_f16(tmem, ad, bd, idesc, kk > 0);
        }
      } else {
        const uint32_t idesc = tc::idesc_f16(true, 128, n, true, true);
        const uint32_t rb = 2 * n;  // bytes per key row of B
        for (int kk = 0; kk < 8; ++kk) {
          uint64_t ad = tc::smem_desc(a0 + kk * 2048, 16384, 1024);
          uint64_t bd = tc::smem_desc(b0 + kk * 16 * rb, 0, 8 * rb, tc::layout_for_row_bytes(rb));
          tc::mma_f16(tmem, ad, bd, idesc, kk > 0);
        }
      }
      tc::mma_commit(&bars[1]);
      ok = tc::mbar_wait(&bars[1], 0, 2000000000ull);
    }
    if (!ok) atomicExch(status, 1);
  }
  __syncthreads();
  tc::tc_fence_after();
  if (*reinterpret_cast<volatile int*>(status) == 0) {
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    const int row = warp * 32 + (tid & 31);
    float v[32];
    for (int c0 = 0; c0 < n; c0 += 32) {
      if (n - c0 >= 32) {
        tc::tmem_ld32(tmem + lane_base + c0, v);
        for (int j = 0; j < 32; ++j) out[(size_t)row * n + c0 + j] = v[j];
      } else {
        tc::tmem_ld16(tmem + lane_base + c0, v);
        for (int j = 0; j < 16; ++j) out[(size_t)row * n + c0 + j] = v[j];
      }
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, 128);
}

}  // namespace
}  // namespace dropkv

using namespace dropkv;

extern "C" int dropkv_selftest_tcgen05(int mode, const void* a, const void* b, int n, float* out,
                                       int* status, void* stream) {
  if (mode < 0 || mode > 5) return fail(DROPKV_ERR_ARG, "selftest mode must be 0..5");
  if (!(n == 16 || n == 32 || n == 64 || n == 128)) return fail(DROPKV_ERR_ARG, "n must be 16, 32, 64 or 128");
  if (!a || !b || !out || !status) return fail(DROPKV_ERR_ARG, "NULL pointer");
  const int D = (mode == 2 || mode == 3) ? 64 : 128;
  const int pv = (mode & 1) || mode >= 4;
  const int mn = mode == 4 ? 1 : (mode == 5 ? 2 : 0);
  if (mode == 4 && n == 128) return fail(DROPKV_ERR_ARG, "mode 4 takes n = 16, 32 or 64");
  if (mode == 5 && n == 16) return fail(DROPKV_ERR_ARG, "mode 5 takes n = 32, 64 or 128");
  CUtensorMap map;
  int rc = make_kv_tensor_map(&map, a, 1, 128, D, true);
  if (rc) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int b_regions = pv ? 2 : D / 64;
  size_t smem = 1024 + 128 * D * 2 + (size_t)b_regions * n * 128 + 64;
  const uint16_t* bb = reinterpret_cast<const uint16_t*>(b);
  if (D == 128) {
    cudaFuncSetAttribute(selftest_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    selftest_kernel<128><<<1, 128, smem, st>>>(map, bb, n, pv, mn, out, status);
  } else {
    cudaFuncSetAttribute(selftest_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    selftest_kernel<64><<<1, 128, smem, st>>>(map, bb, n, pv, mn, out, status);
  }
  return check_launch("selftest_tcgen05");
}
