// Decode attention over the (compressed) KV cache: for every sequence b and query
// head h, O[b, h, i, :] = softmax(scale * Q[b, h, i, :] K[b, h / g, :L, :]^T) V[b, h / g, :L, :]
// with the Lq query rows tail-aligned to the keys (row i sees keys j <= L - Lq + i),
// which is what the model's attention computes over the cache DropKVCache.update
// returns (dropkv_cache.py:609-617 append the token, the model's SDPA attends).
//
// A handful of query rows per KV head make this an HBM-bound stream over K and V.
// The keys of each (sequence, KV head, tile of 8 query rows) are split over CTAs
// of 12 warps, one CTA per SM and all of them in one wave; each warp takes every
// 12th step of 16 keys and keeps a running (max, sum, output) of its own. A
// step's K rows are fetched for the next step as soon as its S is computed, its V
// rows as soon as its P.V is issued, so every warp keeps a step of loads in
// flight.
//
// Both products run on the tensor cores as m16n8k16 MMAs fed straight from
// registers, so no shuffle reduction per key is needed:
//   S  = Q K^T   A = the 8 query rows (rows 8..15 zero), B = K^T: 8 keys per MMA;
//   O^T += V^T P^T   A = V^T (16 columns of D), B = P^T: the softmax weights of the
//                    16 keys, taken from S's accumulator registers as they lie.
// A dot product may sum its D terms in any order, so the D axis is permuted to
// suit the loads: lane (gid, tig) of a warp (gid = lane / 4, tig = lane % 4) reads
// the bytes [64 i + 16 tig, +16) of its key row for K (i < D / 32; four lanes
// cover 64 contiguous bytes of a row) and the bytes [128 i + 16 gid, +16) of four
// key rows for V (eight lanes cover 128 contiguous bytes), every load a 16-byte
// vector of whole 32-byte sectors; the MMA's k-index pairs of Q use the same
// permutation as those of K, and the output columns carry the V permutation back.
//
// The warps' partials are merged in shared memory; the CTAs of one tile write
// theirs (output, max, sum) to the workspace, and the CTA that increments the
// tile's counter last merges them (max-rescaled sum, loads batched), writes O and
// resets the counter, so the workspace is left as it was found. No wait in this
// kernel depends on another CTA.
#include <algorithm>
#include <atomic>
#include <type_traits>

#include "common.cuh"

namespace dropkv {
namespace {

constexpr int DA_WARPS = 12;
constexpr int DA_NT = 32 * DA_WARPS;
constexpr int DA_KS = 16;              // keys per step (the k extent of the P.V MMA)
constexpr int DA_ROWS = 8;             // query rows per tile (the n extent of the P.V MMA)
constexpr int DA_MIN_STEPS = DA_WARPS; // key steps per CTA at least
constexpr int DA_MAX_SPLITS = 256;
constexpr int DA_BATCH = 8;            // partials read at once by the merge

// Dynamic shared memory: the warps' partials, then the merge's factors and sums.
template <int D>
struct DaSmem {
  static constexpr int WO = 0;                                   // float [WARPS][ROWS][D]
  static constexpr int WM = WO + DA_WARPS * DA_ROWS * D * 4;     // float [WARPS][ROWS]
  static constexpr int WL = WM + DA_WARPS * DA_ROWS * 4;         // float [WARPS][ROWS]
  static constexpr int FAC = WL + DA_WARPS * DA_ROWS * 4;        // float [MAX_SPLITS][ROWS]
  static constexpr int LS = FAC + DA_MAX_SPLITS * DA_ROWS * 4;   // float [MAX_SPLITS][ROWS]
  static constexpr int RS = LS + DA_MAX_SPLITS * DA_ROWS * 4;    // float [ROWS]
  static constexpr int BYTES = RS + DA_ROWS * 4 + 16;            // + the last-CTA flag
};

struct DaArgs {
  const void* q;
  int64_t q_sb, q_sh, q_ss, q_sd;
  const void* k;
  const void* v;
  int64_t kv_sb, kv_sh;  // element strides of a sequence and a KV head; rows of D contiguous
  int Hq, Hkv, g, Lq, L;
  int M;                 // g * Lq query rows per (b, KV head)
  int ntiles;            // tiles of 8 query rows per (b, KV head)
  int splits;            // CTAs per tile
  int steps;             // key steps per CTA
  float scale_log2;      // scale * log2(e)
  float* part;           // [tiles][splits][8][D + 4]: output, max, sum (rows of 16-byte multiples)
  unsigned* counter;     // [tiles]
  void* out;             // [B, Hq, Lq, D]
  // keys [pos, L) come from k_new / v_new (rows of D, strides new_sb, new_sh) and
  // are stored into the buffers (k_buf / v_buf, the same memory as k / v) at rows
  // [pos, L) by the first CTA of each (sequence, KV head); pos = L: no new rows
  const void* k_new;
  const void* v_new;
  int64_t new_sb, new_sh;
  int pos;
  void* k_buf;
  void* v_buf;
};

__device__ __forceinline__ uint4 ld_stream(const void* p) {  // read once: no L1 allocation
  uint4 r;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ float ex2(float x) {  // 2^x, hardware approximation; 2^-inf = 0
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <typename T>
__device__ __forceinline__ void mma16816(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  } else {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
}

// two floats rounded to T, x in the low half
template <typename T>
__device__ __forceinline__ uint32_t pack2(float x, float y) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    __nv_bfloat162 h = __floats2bfloat162_rn(x, y);
    return *reinterpret_cast<uint32_t*>(&h);
  } else {
    __half2 h = __floats2half2_rn(x, y);
    return *reinterpret_cast<uint32_t*>(&h);
  }
}

template <typename T>
__device__ __forceinline__ T from_f(float x);
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <>
__device__ __forceinline__ __half from_f<__half>(float x) { return __float2half_rn(x); }

// Column of D held in 32-bit word w of a lane's K slab (lane group tig) and of its
// V slab (lane group gid); the word's second element is the next column.
template <int D>
__device__ __forceinline__ int k_col(int tig, int w) { return 32 * (w >> 2) + 8 * tig + 2 * (w & 3); }
template <int D>
__device__ __forceinline__ int v_col(int gid, int w) { return 64 * (w >> 2) + 8 * gid + 2 * (w & 3); }

template <typename T, int D>
__global__ void __launch_bounds__(DA_NT, 1) decode_attn_kernel(DaArgs a) {
  constexpr int NK = D / 32;  // 16-byte loads per K row and lane
  constexpr int KW = 4 * NK;  // K words per row and lane (two per QK^T k-step)
  constexpr int NV = D / 64;  // 16-byte loads per V row and lane
  constexpr int DT = D / 16;  // P.V MMAs per key step (16 columns of D each)
  constexpr int PR = D + 4;   // floats per row of a partial
  static_assert(DT == 4 * NV, "one V word per column tile");
  using Sm = DaSmem<D>;
  extern __shared__ __align__(16) uint8_t smem[];
  float(*wo)[DA_ROWS][D] = reinterpret_cast<float(*)[DA_ROWS][D]>(smem + Sm::WO);
  float(*wm)[DA_ROWS] = reinterpret_cast<float(*)[DA_ROWS]>(smem + Sm::WM);
  float(*wl)[DA_ROWS] = reinterpret_cast<float(*)[DA_ROWS]>(smem + Sm::WL);
  float(*fac)[DA_ROWS] = reinterpret_cast<float(*)[DA_ROWS]>(smem + Sm::FAC);
  float(*lsh)[DA_ROWS] = reinterpret_cast<float(*)[DA_ROWS]>(smem + Sm::LS);
  float* rsum = reinterpret_cast<float*>(smem + Sm::RS);
  int* last_cta = reinterpret_cast<int*>(smem + Sm::RS + DA_ROWS * 4);

  const int split = blockIdx.x, bh = blockIdx.y, tile = blockIdx.z;
  const int b = bh / a.Hkv, hkv = bh % a.Hkv;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gid = lane >> 2, tig = lane & 3;
  const int m0 = tile * DA_ROWS, mvalid = min(DA_ROWS, a.M - m0);
  const T* kb = reinterpret_cast<const T*>(a.k) + b * a.kv_sb + hkv * a.kv_sh;
  const T* vb = reinterpret_cast<const T*>(a.v) + b * a.kv_sb + hkv * a.kv_sh;
  // rows from pos on: the new rows (not yet in the buffers)
  const T* knb = reinterpret_cast<const T*>(a.k_new) + b * a.new_sb + hkv * a.new_sh - (int64_t)a.pos * D;
  const T* vnb = reinterpret_cast<const T*>(a.v_new) + b * a.new_sb + hkv * a.new_sh - (int64_t)a.pos * D;
  // launched with programmatic dependent launch: every global access below waits
  // for the kernel before this one (it may write Q, the new rows or reuse the
  // workspace); the next kernel may be scheduled as this one's CTAs exit
  pdl_launch_dependents();
  pdl_wait();
  if (a.pos < a.L && split == 0 && tile == 0) {  // append the new rows to the buffers (read from the inputs here)
    const int nvec = (a.L - a.pos) * D / 8;
    uint4* kd = reinterpret_cast<uint4*>(reinterpret_cast<T*>(a.k_buf) + b * a.kv_sb + hkv * a.kv_sh + (int64_t)a.pos * D);
    uint4* vd = reinterpret_cast<uint4*>(reinterpret_cast<T*>(a.v_buf) + b * a.kv_sb + hkv * a.kv_sh + (int64_t)a.pos * D);
    const uint4* ks = reinterpret_cast<const uint4*>(knb + (int64_t)a.pos * D);
    const uint4* vs = reinterpret_cast<const uint4*>(vnb + (int64_t)a.pos * D);
    for (int e = threadIdx.x; e < nvec; e += DA_NT) {
      kd[e] = ks[e];
      vd[e] = vs[e];
    }
  }
  const int j_begin = split * a.steps * DA_KS;
  const int j_end = min(a.L, j_begin + a.steps * DA_KS);

  // query row gid of the tile, in the K permutation: qa[w] holds columns
  // k_col(tig, w) and k_col(tig, w) + 1
  uint32_t qa[KW];
  int bound = -1;  // last key this row sees (-1: a padding row)
  {
    const int m = m0 + gid;
    if (gid < mvalid) {
      const int h = hkv * a.g + m / a.Lq, qi = m % a.Lq;
      bound = a.L - a.Lq + qi;
      const uint16_t* qp = reinterpret_cast<const uint16_t*>(a.q) + b * a.q_sb + h * a.q_sh + qi * a.q_ss;
#pragma unroll
      for (int w = 0; w < KW; ++w) {
        const int d = k_col<D>(tig, w);
        qa[w] = (uint32_t)qp[d * a.q_sd] | ((uint32_t)qp[(d + 1) * a.q_sd] << 16);
      }
    } else {
#pragma unroll
      for (int w = 0; w < KW; ++w) qa[w] = 0u;
    }
  }

  float o[DT][4];
#pragma unroll
  for (int t = 0; t < DT; ++t) o[t][0] = o[t][1] = o[t][2] = o[t][3] = 0.f;
  float mrun = -INFINITY, lrun = 0.f;  // row gid: running max (base 2) and this lane's share of the sum

  // K rows j0 + gid and j0 + 8 + gid (this lane's slab of each), V rows
  // j0 + 2 tig + {0, 1, 8, 9} (this lane's columns of each); rows past the CTA's
  // keys read as zeros
  uint4 kr[2][NK], vr[4][NV];
  auto load_k = [&](int j0) {
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const int j = j0 + 8 * nt + gid;
#pragma unroll
      for (int i = 0; i < NK; ++i)
        kr[nt][i] = j < j_end ? ld_stream((j < a.pos ? kb : knb) + (int64_t)j * D + 32 * i + 8 * tig)
                              : make_uint4(0u, 0u, 0u, 0u);
    }
  };
  auto load_v = [&](int j0) {
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int j = j0 + 2 * tig + (r & 1) + 8 * (r >> 1);
#pragma unroll
      for (int i = 0; i < NV; ++i)
        vr[r][i] = j < j_end ? ld_stream((j < a.pos ? vb : vnb) + (int64_t)j * D + 64 * i + 8 * gid)
                              : make_uint4(0u, 0u, 0u, 0u);
    }
  };
  const int jstep = DA_WARPS * DA_KS;
  int j0 = j_begin + warp * DA_KS;
  if (j0 < j_end) {
    load_k(j0);
    load_v(j0);
  }
  for (; j0 < j_end; j0 += jstep) {
    const int jn = j0 + jstep;
    // S = Q K^T for the 16 keys: s[nt][e] = S[row gid][key j0 + 8 nt + 2 tig + e] (e < 2)
    float s[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
      const uint32_t* kw = reinterpret_cast<const uint32_t*>(kr[nt]);
#pragma unroll
      for (int ks = 0; ks < KW / 2; ++ks) mma16816<T>(s[nt], qa[2 * ks], 0u, qa[2 * ks + 1], 0u, kw[2 * ks], kw[2 * ks + 1]);
    }
    if (jn < j_end) load_k(jn);  // the next step's K, in flight during this step's softmax and P.V
    // online softmax of row gid (base 2); masked keys get -inf, hence weight 0
    float x[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int j = j0 + 8 * (e >> 1) + 2 * tig + (e & 1);
      x[e] = (j < j_end && j <= bound) ? s[e >> 1][e & 1] * a.scale_log2 : -INFINITY;
    }
    float mx = fmaxf(fmaxf(x[0], x[1]), fmaxf(x[2], x[3]));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float mnew = fmaxf(mrun, mx);
    const float muse = mnew == -INFINITY ? 0.f : mnew;
    const float alpha = ex2(mrun - muse);
    float p[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) p[e] = ex2(x[e] - muse);
    lrun = lrun * alpha + ((p[0] + p[1]) + (p[2] + p[3]));
    mrun = mnew;
    // this lane's output columns belong to rows 2 tig and 2 tig + 1
    const float a_lo = __shfl_sync(0xffffffffu, alpha, 8 * tig);
    const float a_hi = __shfl_sync(0xffffffffu, alpha, 8 * tig + 4);
    const uint32_t pb0 = pack2<T>(p[0], p[1]), pb1 = pack2<T>(p[2], p[3]);
    uint32_t va[DT][4];  // A = V^T: rows v_col(gid, t) and v_col(gid, t) + 1, keys 2 tig + {0, 1, 8, 9}
    {
      const uint32_t* v0 = reinterpret_cast<const uint32_t*>(vr[0]);
      const uint32_t* v1 = reinterpret_cast<const uint32_t*>(vr[1]);
      const uint32_t* v2 = reinterpret_cast<const uint32_t*>(vr[2]);
      const uint32_t* v3 = reinterpret_cast<const uint32_t*>(vr[3]);
#pragma unroll
      for (int t = 0; t < DT; ++t) {
        va[t][0] = __byte_perm(v0[t], v1[t], 0x5410);
        va[t][1] = __byte_perm(v0[t], v1[t], 0x7632);
        va[t][2] = __byte_perm(v2[t], v3[t], 0x5410);
        va[t][3] = __byte_perm(v2[t], v3[t], 0x7632);
      }
    }
    if (jn < j_end) load_v(jn);  // the next step's V
#pragma unroll
    for (int t = 0; t < DT; ++t) {
      o[t][0] *= a_lo;
      o[t][1] *= a_hi;
      o[t][2] *= a_lo;
      o[t][3] *= a_hi;
      mma16816<T>(o[t], va[t][0], va[t][1], va[t][2], va[t][3], pb0, pb1);
    }
  }

  // ---- the CTA's partial: warps merged through shared memory -----------------
  lrun += __shfl_xor_sync(0xffffffffu, lrun, 1);
  lrun += __shfl_xor_sync(0xffffffffu, lrun, 2);
  if (tig == 0) {
    wm[warp][gid] = mrun;
    wl[warp][gid] = lrun;
  }
#pragma unroll
  for (int t = 0; t < DT; ++t) {
    const int d = v_col<D>(gid, t);
    wo[warp][2 * tig][d] = o[t][0];
    wo[warp][2 * tig + 1][d] = o[t][1];
    wo[warp][2 * tig][d + 1] = o[t][2];
    wo[warp][2 * tig + 1][d + 1] = o[t][3];
  }
  __syncthreads();
  if (tid < DA_ROWS) {  // per row: the warps' factors (fac[w][r]), the CTA's max and sum
    float mm = -INFINITY;
#pragma unroll
    for (int w = 0; w < DA_WARPS; ++w) mm = fmaxf(mm, wm[w][tid]);
    float l = 0.f;
#pragma unroll
    for (int w = 0; w < DA_WARPS; ++w) {
      const float f = mm == -INFINITY ? 0.f : ex2(wm[w][tid] - mm);
      fac[w][tid] = f;
      l = fmaf(f, wl[w][tid], l);
    }
    lsh[0][tid] = mm;
    rsum[tid] = l;
  }
  __syncthreads();
  const int tile_id = bh * a.ntiles + tile;
  T* op = reinterpret_cast<T*>(a.out);
  auto out_at = [&](int r, int d) -> T* {
    const int m = m0 + r, h = hkv * a.g + m / a.Lq, qi = m % a.Lq;
    return op + (((size_t)b * a.Hq + h) * a.Lq + qi) * D + d;
  };
  auto cta_out = [&](int r, int d) {
    float acc = 0.f;
#pragma unroll
    for (int w = 0; w < DA_WARPS; ++w) acc = fmaf(fac[w][r], wo[w][r][d], acc);
    return acc;
  };
  if (a.splits == 1) {  // the only CTA of the tile: O directly
    for (int e = tid; e < mvalid * D; e += DA_NT) {
      const int r = e / D, d = e % D;
      *out_at(r, d) = from_f<T>(rsum[r] > 0.f ? cta_out(r, d) / rsum[r] : 0.f);
    }
    return;
  }
  float* pp = a.part + ((size_t)tile_id * a.splits + split) * DA_ROWS * PR;
  for (int e = tid; e < mvalid * D; e += DA_NT) {
    const int r = e / D, d = e % D;
    pp[r * PR + d] = cta_out(r, d);
  }
  if (tid < mvalid) {
    pp[tid * PR + D] = lsh[0][tid];
    pp[tid * PR + D + 1] = rsum[tid];
  }
  // ---- the last CTA of the tile merges every partial ---------------------------
  // the arrival is an acquire-release add: it publishes this CTA's partial (its
  // threads' stores come before it through the barrier) and, in the last CTA,
  // acquires every other CTA's; the barrier after it orders this CTA's loads
  __syncthreads();
  if (tid == 0) {
    unsigned prev;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(prev) : "l"(&a.counter[tile_id]) : "memory");
    *last_cta = prev == (unsigned)(a.splits - 1);
  }
  __syncthreads();
  if (!*last_cta) return;
  const float* pt = a.part + (size_t)tile_id * a.splits * DA_ROWS * PR;
  // (a) every partial's max and sum into shared memory
  for (int i = tid; i < a.splits * mvalid; i += DA_NT) {
    const int s2 = i / mvalid, r = i % mvalid;
    const float* ps = pt + ((size_t)s2 * DA_ROWS + r) * PR + D;
    fac[s2][r] = __ldcg(ps);
    lsh[s2][r] = __ldcg(ps + 1);
  }
  __syncthreads();
  // (b) one warp per row: the row's max, each partial's factor, the total sum
  if (warp < mvalid) {
    const int r = warp;
    float mm = -INFINITY;
    for (int s2 = lane; s2 < a.splits; s2 += 32) mm = fmaxf(mm, fac[s2][r]);
#pragma unroll
    for (int o2 = 16; o2 > 0; o2 >>= 1) mm = fmaxf(mm, __shfl_xor_sync(0xffffffffu, mm, o2));
    float l = 0.f;
    for (int s2 = lane; s2 < a.splits; s2 += 32) {
      const float f = mm == -INFINITY ? 0.f : ex2(fac[s2][r] - mm);
      fac[s2][r] = f;
      l = fmaf(f, lsh[s2][r], l);
    }
#pragma unroll
    for (int o2 = 16; o2 > 0; o2 >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o2);
    if (lane == 0) rsum[r] = l;
  }
  __syncthreads();
  // (c) O, four columns per thread, DA_BATCH partials loaded at a time
  for (int e = tid; e < mvalid * (D / 4); e += DA_NT) {
    const int r = e / (D / 4), d = 4 * (e % (D / 4));
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s0 = 0; s0 < a.splits; s0 += DA_BATCH) {
      float4 vv[DA_BATCH];
#pragma unroll
      for (int u = 0; u < DA_BATCH; ++u)
        vv[u] = s0 + u < a.splits
                    ? __ldcg(reinterpret_cast<const float4*>(pt + ((size_t)(s0 + u) * DA_ROWS + r) * PR + d))
                    : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int u = 0; u < DA_BATCH; ++u) {
        const float f = s0 + u < a.splits ? fac[s0 + u][r] : 0.f;
        acc.x = fmaf(f, vv[u].x, acc.x);
        acc.y = fmaf(f, vv[u].y, acc.y);
        acc.z = fmaf(f, vv[u].z, acc.z);
        acc.w = fmaf(f, vv[u].w, acc.w);
      }
    }
    const float inv = rsum[r] > 0.f ? 1.f / rsum[r] : 0.f;
    T* dst = out_at(r, d);
    dst[0] = from_f<T>(acc.x * inv);
    dst[1] = from_f<T>(acc.y * inv);
    dst[2] = from_f<T>(acc.z * inv);
    dst[3] = from_f<T>(acc.w * inv);
  }
  if (tid == 0) a.counter[tile_id] = 0u;  // ready for the next launch on this workspace
}

using DaKernel = void (*)(DaArgs);

int da_num_sms() {
  static std::atomic<int> cache[64];  // zero: not queried yet
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64) {
    const int c = cache[dev].load(std::memory_order_relaxed);
    if (c > 0) return c;
  }
  int n = 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n < 1) {
    cudaGetLastError();
    n = 148;
  }
  if (dev >= 0 && dev < 64) cache[dev].store(n, std::memory_order_relaxed);
  return n;
}

struct DaPlan {
  int ntiles, tiles, splits, steps;
  size_t off_counter, off_part, bytes;
};

// CTAs per tile: as many as keep the launch to one CTA per SM (one wave), each
// with at least DA_MIN_STEPS key steps; the last CTA never starts empty.
DaPlan plan_da(int B, int Hkv, int M, int L, int D) {
  DaPlan p;
  p.ntiles = (M + DA_ROWS - 1) / DA_ROWS;
  p.tiles = B * Hkv * p.ntiles;
  const int nsteps = (L + DA_KS - 1) / DA_KS;
  int splits = std::max(1, std::min(da_num_sms() / p.tiles, (nsteps + DA_MIN_STEPS - 1) / DA_MIN_STEPS));
  splits = std::min(splits, DA_MAX_SPLITS);
  p.steps = (nsteps + splits - 1) / splits;
  p.splits = (nsteps + p.steps - 1) / p.steps;
  p.off_counter = 256;  // the first 256 bytes: the status word (always zero here)
  p.off_part = align_up(p.off_counter + (size_t)p.tiles * 4, 256);
  p.bytes = p.splits > 1 ? p.off_part + (size_t)p.tiles * p.splits * DA_ROWS * (D + 4) * 4 : p.off_part;
  return p;
}

}  // namespace

size_t decode_attention_workspace_size(int B, int Hq, int Hkv, int Lq, int L, int D) {
  return plan_da(B, Hkv, (Hq / Hkv) * Lq, L, D).bytes;
}

int launch_decode_attention(const void* q, int64_t q_sb, int64_t q_sh, int64_t q_ss, int64_t q_sd, int Lq,
                            const void* k, const void* v, int64_t kv_sb, int64_t kv_sh, int dtype, int B, int Hq,
                            int Hkv, int L, int D, float scale, void* out, void* ws, cudaStream_t st,
                            const void* k_new, const void* v_new, int64_t new_sb, int64_t new_sh, int pos) {
  DaArgs a;
  a.k_new = k_new;
  a.v_new = v_new;
  a.new_sb = new_sb;
  a.new_sh = new_sh;
  a.pos = k_new ? pos : L;
  a.k_buf = const_cast<void*>(k);
  a.v_buf = const_cast<void*>(v);
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
  const DaPlan p = plan_da(B, Hkv, a.M, L, D);
  if (p.ntiles > 65535) return fail(DROPKV_ERR_UNSUPPORTED, "decode attention: %d query rows per KV head", a.M);
  a.ntiles = p.ntiles;
  a.splits = p.splits;
  a.steps = p.steps;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.counter = reinterpret_cast<unsigned*>(static_cast<uint8_t*>(ws) + p.off_counter);
  a.part = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + p.off_part);
  a.out = out;
  DaKernel kern;
  const int var = (dtype == DROPKV_DTYPE_BF16 ? 0 : 2) + (D == 128 ? 0 : 1);
  if (dtype == DROPKV_DTYPE_BF16)
    kern = D == 128 ? decode_attn_kernel<__nv_bfloat16, 128> : decode_attn_kernel<__nv_bfloat16, 64>;
  else
    kern = D == 128 ? decode_attn_kernel<__half, 128> : decode_attn_kernel<__half, 64>;
  const int smem = D == 128 ? DaSmem<128>::BYTES : DaSmem<64>::BYTES;
  static DeviceOnce done[4];  // shared-memory attribute set, per variant and device
  int dev = 0;
  cudaGetDevice(&dev);
  if (!done[var].done(dev)) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
      return fail(DROPKV_ERR_CUDA, "cannot set decode attention shared memory size %d", smem);
    done[var].mark(dev);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.splits, B * Hkv, p.ntiles);
  cfg.blockDim = dim3(DA_NT);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // may start as the previous kernel ends
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a);
  if (e != cudaSuccess) return fail(DROPKV_ERR_CUDA, "decode attention launch: %s", cudaGetErrorString(e));
  return check_launch("decode_attention");
}

}  // namespace dropkv
