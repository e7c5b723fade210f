// Fused tensor-core DropKV scorer for sm_100a (bf16 / fp16 inputs, D in {64, 128},
// M = g*W <= 64 query rows per KV head).
//
// One persistent cooperative launch, one CTA per SM.  CTAs form `groups` groups
// of `gs` CTAs; group g scores heads g, g + groups, ... one round at a time, and
// CTA `rank` of a group owns a contiguous range of <= tmax 128-key tiles of the
// round's head.  Warp roles inside a CTA (coupled only through mbarriers):
//   warp 16     TMA producer: K, V, V tiles of every round into an NS-slot ring;
//   warp 17     MMA issuer (one thread) and TMEM owner;
//   warps 0-15  epilogue: warp w reads TMEM lanes 32*(w%4).. (32 keys of a tile)
//               and query columns [(w/4)*N/4, (w/4+1)*N/4).
// Per head and CTA:
//
//   pass 1  K tiles stream in by TMA (L2 evict-first); tcgen05 computes the logit
//           tile S = K Q^T (keys on the MMA M axis, the M query rows on N) into
//           TMEM, where it stays for pass 2.  The CTA-local softmax max m and sum s
//           per query row follow from the TMEM tiles; p = exp(l - m) is split into
//           bf16/fp16 hi + lo halves in shared memory (MN-major: a row per key) and
//           V tiles (TMA, L2 evict-last so pass 2 finds them in L2) give
//           y^T += V^T p_hi^T + V^T p_lo^T (fp32 accumulation in TMEM: y keeps
//           ~16 mantissa bits of p).  The partial (m, s, y) goes to global memory.
//   merge   group barrier; each CTA merges a 1/gs slice of the head's M x D
//           elements of y with the max-rescale rule (dropkv_triton.py:441-452),
//           plus lse; group barrier.
//   pass 2  y is split hi + lo into shared memory; V tiles come back by TMA
//           (L2 hits); tcgen05 gives <v_j, y_m> = V (y_hi + y_lo)^T in TMEM; the
//           epilogue forms ||v_j||^2 from the V tile still in the ring, and
//           p = exp(l - lse) clamped to [0,1] (rounded to the input dtype when
//           requested), w = (p / (1 - p + eps))^2 and
//           score_j = (sum w ||v_j||^2 - 2 sum w <v_j,y_m> + sum w ||y_m||^2) / g,
//           the reference's termA - termB + termC (dropkv_triton.py:94-108); the
//           four column groups of a key combine their sums in a fixed order.
//
// Group barriers are bounded spins on global counters (zeroed by the host before
// the launch); every wait in the kernel gives up after a timeout, records a
// device status and lets the CTA run to its end without further waits, so a
// fault in this logic ends the kernel instead of hanging the GPU.
#include <atomic>
#include <cmath>
#include <mutex>
#include <cstring>
#include <type_traits>

#include "tc_common.cuh"

namespace dropkv {

// ---------------------------------------------------------------------------
// Tensor map (host)
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  // looked up once per process (a function-local static: initialised by one thread)
  static const EncodeTiledFn fn = []() -> EncodeTiledFn {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<EncodeTiledFn>(p);
    return nullptr;
  }();
  return fn;
}

int make_kv_tensor_map(CUtensorMap* map, const void* base, int BH, int L, int D, bool bf16, int64_t head_stride) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(DROPKV_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
  if (reinterpret_cast<uintptr_t>(base) % 16) return fail(DROPKV_ERR_ARG, "K/V must be 16-byte aligned");
  const int64_t hs = head_stride ? head_stride : (int64_t)L * D;
  if ((hs * 2) % 16) return fail(DROPKV_ERR_ARG, "K/V head stride must be a multiple of 8 elements");
  cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)L, (cuuint64_t)BH};
  cuuint64_t strides[2] = {(cuuint64_t)D * 2, (cuuint64_t)hs * 2};
  cuuint32_t box[3] = {64, 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                  const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(DROPKV_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return DROPKV_OK;
}

int make_kv_tensor_map_4d(CUtensorMap* map, const void* base, int B, int Hkv, int L, int D, bool bf16, int64_t sb,
                          int64_t sh, int64_t ss) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(DROPKV_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
  if (reinterpret_cast<uintptr_t>(base) % 16) return fail(DROPKV_ERR_ARG, "K/V must be 16-byte aligned");
  if ((sb * 2) % 16 || (sh * 2) % 16 || (ss * 2) % 16)
    return fail(DROPKV_ERR_ARG, "K/V strides must be multiples of 8 elements");
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)L, (cuuint64_t)Hkv, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)ss * 2, (cuuint64_t)sh * 2, (cuuint64_t)sb * 2};
  cuuint32_t box[4] = {64, 128, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                  const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(DROPKV_ERR_CUDA, "cuTensorMapEncodeTiled (4-D K/V) failed (%d)", (int)r);
  return DROPKV_OK;
}

// Q viewed as {D, Lq, Hq, B} with box {64, W, g, 1}: one load per 64-wide slab
// brings the W window rows of the g query heads of one KV head, in the order of
// the scorer's query rows (m = head * W + row), under the 128-byte swizzle.
// Only for Q with unit element stride and 16-byte aligned base and strides;
// returns false (and encodes nothing) otherwise.
bool make_q_tensor_map(CUtensorMap* map, const ScoreProblem& p, bool bf16) {
  EncodeTiledFn fn = encode_fn();
  if (!fn || p.q_sd != 1 || (p.D % 64) || p.W > 256 || p.g > 256) return false;
  const int64_t sb[3] = {p.q_ss * 2, p.q_sh * 2, p.q_sb * 2};
  if (reinterpret_cast<uintptr_t>(p.q) % 16) return false;
  for (int i = 0; i < 3; ++i)
    if (sb[i] <= 0 || sb[i] % 16 || sb[i] >= (int64_t(1) << 40)) return false;
  cuuint64_t dims[4] = {(cuuint64_t)p.D, (cuuint64_t)p.Lq, (cuuint64_t)p.Hq, (cuuint64_t)p.B};
  cuuint64_t strides[3] = {(cuuint64_t)sb[0], (cuuint64_t)sb[1], (cuuint64_t)sb[2]};
  cuuint32_t box[4] = {64, (cuuint32_t)p.W, (cuuint32_t)p.g, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                  const_cast<void*>(p.q), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

namespace {

constexpr int TK = 128;                      // keys per tile = MMA M
constexpr int NEPI = 512;                    // epilogue threads (warps 0-15)
constexpr int NEW = NEPI / 32;               // epilogue warps
constexpr int NTH = NEPI + 64;               // + TMA producer warp + MMA warp
constexpr int WARP_TMA = NEW, WARP_MMA = NEW + 1;
// Waits for the hardware's own completions (in-flight TMA copies, committed MMAs)
// give up after 1 s; waits on other roles and on other CTAs use TcArgs::wait_ns
// (1 s unless a test shortens it).
constexpr uint64_t kWaitNs = 1000000000ull;
constexpr int kMaxGs = 256;                  // CTAs per head group (at most)
constexpr int kWts = 1024;                   // merge maxima / sums buffers (floats each)
constexpr int kMaxTiles = 30;                // TMEM logit tiles per CTA and head (N = 16)
constexpr int kVnWarps = 4;                  // epilogue warps that read a pass-1 V tile for ||v||^2
// Odd groups start this long (per tile of a CTA's range) after the even ones:
// about half a round, so that one half of the SMs streams K and V from HBM while
// the other half runs its L2-only merge and pass 2, instead of all streaming at
// once and then all leaving HBM idle. Measured on the 128K layer (4 rounds) the
// overlap saves ~3 us a round, less than the offset costs once; so only launches
// with many rounds (kStaggerRounds or more) stagger.
constexpr uint64_t kStaggerNsPerTile = 1250;
constexpr int kStaggerRounds = 8;

struct TcArgs {
  ScoreProblem p;
  int BH;
  int gs, groups, rounds, tiles, tmax;
  int tmax_cta;  // tiles of the largest CTA range
  float c;       // log2(e) / sqrt(D): logits in the base-2 domain
  float pscale;  // scale of p before the hi/lo split (2^15 for fp16, 1 for bf16)
  int* ctr;      // [2 * BH] group-barrier counters (zero at launch)
  float* part_m; // [BH][gs][M]  (base-2 max)
  float* part_s; // [BH][gs][M]
  float* part_y; // [BH][gs][M][D]
  float* y_g;    // [BH][M][D]
  float* lse_g;  // [BH][M]      (base-2)
  int* status;   // device status word (0 = ok)
  int q_tma;     // 1: the TMA warp loads the Q window (qmap), 0: the epilogue stages it
  unsigned long long* trace;  // per CTA and round: globaltimer at phase ends
  uint64_t wait_ns;  // limit of a wait on another role or CTA, then status + abort
};

// Phase timestamps recorded by epilogue thread 0 of every CTA (ns, globaltimer):
// trace[3 + (cta * rounds + round) * kTraceEv + ev]; trace[0..2] = {ctas, rounds, kTraceEv}.
enum { TR_START, TR_LOGITS, TR_MAX, TR_PV, TR_BAR_A, TR_MERGE, TR_BAR_B, TR_YSTAGE, TR_PASS2, kTraceEv };

// mbarrier indices after full[NS], free[NS] and s_done[kMaxTiles]
enum {
  B_QREADY = 0, B_PREADY0, B_PREADY1, B_PFREE0, B_PFREE1, B_YDONE, B_YREADY,
  B_S2READY0, B_S2READY1, B_S2FREE0, B_S2FREE1, B_FIN, kAuxBars
};

// Shared-memory layout.  Q and y are K-major SW128 operands (NPAD rows of 64
// elements per 128-byte region row); P tiles are MN-major: one row per key holding
// its NPAD query columns (2 * NPAD bytes, swizzled at that width), which is the
// layout an epilogue thread owning one key writes with vector stores.
template <int D, int NPAD, int NS, int NPB>
struct Lay {
  static constexpr int TILE = TK * D * 2;         // one K or V tile
  static constexpr int RB = NPAD * 128;           // one SW128 region of NPAD rows
  static constexpr int PRB = 2 * NPAD;            // bytes per key row of a P tile
  static constexpr int PT = TK * PRB;             // one P tile (hi or lo half)
  static constexpr int TMAX = (512 - 2 * NPAD) / NPAD;
  static constexpr int RING = 0;
  static constexpr int QS = RING + NS * TILE;     // D/64 regions
  static constexpr int PS = QS + (D / 64) * RB;   // [NPB buffers][hi/lo] P tiles
  static constexpr int YS = PS + NPB * 2 * PT;    // [D/64][hi/lo] regions (hi and lo rows stacked)
  static constexpr int FL = YS + 2 * (D / 64) * RB;
  static constexpr int MLOC = FL;                 // floats [NPAD]
  static constexpr int LSE = MLOC + 4 * NPAD;
  static constexpr int YN = LSE + 4 * NPAD;
  static constexpr int BND = YN + 4 * NPAD;       // int [NPAD] causal bound per row
  static constexpr int RED = BND + 4 * NPAD;      // [4 lane quadrants][NPAD]
  static constexpr int XCH = RED + 16 * NPAD;     // [2 buf][3 column groups][3 sums][TK]
  static constexpr int VN = XCH + 4 * 18 * TK;    // [TMAX][TK] ||v||^2 of the CTA's keys
  static constexpr int WTS = VN + 4 * TMAX * TK;  // [2][kWts]
  static constexpr int BAR = WTS + 8 * kWts;      // mbarriers
  static constexpr int NBAR = 2 * NS + kMaxTiles + kAuxBars;
  static constexpr int MISC = BAR + 8 * NBAR;     // tmem slot, flags
  static constexpr int BYTES = MISC + 64;
  static constexpr int ALLOC = BYTES + 1024;      // + alignment slack
};

template <typename T>
__device__ __forceinline__ uint16_t to_bits(float x);
template <>
__device__ __forceinline__ uint16_t to_bits<__nv_bfloat16>(float x) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(x));
}
template <>
__device__ __forceinline__ uint16_t to_bits<__half>(float x) {
  return __half_as_ushort(__float2half_rn(x));
}
template <typename T>
__device__ __forceinline__ float from_bits(uint16_t b);
template <>
__device__ __forceinline__ float from_bits<__nv_bfloat16>(uint16_t b) {
  return __bfloat162float(__ushort_as_bfloat16(b));
}
template <>
__device__ __forceinline__ float from_bits<__half>(uint16_t b) {
  return __half2float(__ushort_as_half(b));
}

// Two floats rounded to T and packed (x in the low half), and back.
template <typename T>
__device__ __forceinline__ uint32_t pack2(float x, float y);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float x, float y) {
  __nv_bfloat162 h = __floats2bfloat162_rn(x, y);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float x, float y) {
  __half2 h = __floats2half2_rn(x, y);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <typename T>
__device__ __forceinline__ float2 unpack2(uint32_t u);
template <>
__device__ __forceinline__ float2 unpack2<__nv_bfloat16>(uint32_t u) {
  return __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&u));
}
template <>
__device__ __forceinline__ float2 unpack2<__half>(uint32_t u) {
  return __half22float2(*reinterpret_cast<__half2*>(&u));
}

// p rounded to the input dtype (p in [0, 1], finite).  bf16 round-to-nearest-even
// is done on the integer pipe: add 0x7fff plus the lowest kept bit, clear the 16
// dropped bits (exact for finite non-negative inputs); this keeps the conversion
// unit, which also serves exp2 and the reciprocal, free.
// 2^x by the hardware approximation (relative error ~2^-22; results below 2^-126
// flush to zero, far below any weight that reaches a score).
__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <int ROUND>
__device__ __forceinline__ float round_p_t(float p) {
  if (ROUND == DROPKV_ROUND_BF16) {
    const uint32_t u = __float_as_uint(p);
    return __uint_as_float((u + 0x7fffu + ((u >> 16) & 1u)) & 0xffff0000u);
  }
  if (ROUND == DROPKV_ROUND_F16) return __half2float(__float2half_rn(p));
  return p;
}

// Paired fp32 arithmetic: one instruction for both lanes of a float2 (sm_100),
// each lane rounded as the scalar instruction would round it.
__device__ __forceinline__ float2 f2_fma(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n.reg .b64 ra, rb, rc, rd;\nmov.b64 ra, {%2, %3};\nmov.b64 rb, {%4, %5};\nmov.b64 rc, {%6, %7};\n"
      "fma.rn.f32x2 rd, ra, rb, rc;\nmov.b64 {%0, %1}, rd;\n}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
__device__ __forceinline__ float2 f2_add(float2 a, float2 b) {
  float2 d;
  asm("{\n.reg .b64 ra, rb, rd;\nmov.b64 ra, {%2, %3};\nmov.b64 rb, {%4, %5};\n"
      "add.rn.f32x2 rd, ra, rb;\nmov.b64 {%0, %1}, rd;\n}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 f2_sub(float2 a, float2 b) {
  float2 d;
  asm("{\n.reg .b64 ra, rb, rd;\nmov.b64 ra, {%2, %3};\nmov.b64 rb, {%4, %5};\n"
      "sub.rn.f32x2 rd, ra, rb;\nmov.b64 {%0, %1}, rd;\n}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 f2_mul(float2 a, float2 b) {
  float2 d;
  asm("{\n.reg .b64 ra, rb, rd;\nmov.b64 ra, {%2, %3};\nmov.b64 rb, {%4, %5};\n"
      "mul.rn.f32x2 rd, ra, rb;\nmov.b64 {%0, %1}, rd;\n}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
// 1/x by the hardware approximation (x here is in [eps, 1 + eps]).
__device__ __forceinline__ float rcpf(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// Two p rounded to the input dtype, as round_p_t does for one.
template <int ROUND>
__device__ __forceinline__ float2 round_p2(float2 p) {
  if (ROUND == DROPKV_ROUND_BF16) {
    uint32_t u;  // RNE of both in one conversion: x in the upper half, y in the lower
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(u) : "f"(p.x), "f"(p.y));
    return make_float2(__uint_as_float(u & 0xffff0000u), __uint_as_float(u << 16));
  }
  if (ROUND == DROPKV_ROUND_F16) return __half22float2(__floats2half2_rn(p.x, p.y));
  return p;
}

// C columns per lane (C a power of two <= 32): lane l returns column (l % C)
// reduced over all 32 lanes.  log2(C) transpose steps, then the remaining lanes.
template <int C, bool MAX>
__device__ __forceinline__ float col_reduce(float (&v)[C], int lane) {
#pragma unroll
  for (int s = C / 2; s >= 1; s >>= 1) {
    const bool upper = (lane & s) != 0;
#pragma unroll
    for (int i = 0; i < s; ++i) {
      const float send = upper ? v[i] : v[i + s];
      const float keep = upper ? v[i + s] : v[i];
      const float recv = __shfl_xor_sync(0xffffffffu, send, s);
      v[i] = MAX ? fmaxf(keep, recv) : keep + recv;
    }
  }
  float r = v[0];
#pragma unroll
  for (int s = C; s < 32; s <<= 1) {
    const float o = __shfl_xor_sync(0xffffffffu, r, s);
    r = MAX ? fmaxf(r, o) : r + o;
  }
  return r;
}

// TMEM -> registers, C fp32 columns of this thread's lane (C in {4, 8, 16}).
template <int C>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, float* v);
template <>
__device__ __forceinline__ void tmem_ld<16>(uint32_t taddr, float* v) { tc::tmem_ld16(taddr, v); }
template <>
__device__ __forceinline__ void tmem_ld<8>(uint32_t taddr, float* v) { tc::tmem_ld8(taddr, v); }
template <>
__device__ __forceinline__ void tmem_ld<4>(uint32_t taddr, float* v) { tc::tmem_ld4(taddr, v); }

__device__ __forceinline__ void epi_sync() {  // named barrier of the epilogue threads
  asm volatile("bar.sync 1, %0;" ::"r"(NEPI) : "memory");
}
__device__ __forceinline__ void quad_sync(int q) {  // the four warps of TMEM lane quadrant q
  asm volatile("bar.sync %0, 128;" ::"r"(2 + q) : "memory");
}

// HC query columns of one key as hi/lo halves of T, stored to the MN-major P tiles.
template <typename T, int HC, int PRB>
__device__ __forceinline__ void store_p(uint8_t* hi_tile, uint8_t* lo_tile, int jkey, int cbase,
                                        const float (&ps)[HC]) {
  uint32_t hw[HC / 2], lw[HC / 2];
#pragma unroll
  for (int j = 0; j < HC; j += 2) {
    hw[j / 2] = pack2<T>(ps[j], ps[j + 1]);
    const float2 lo = f2_sub(make_float2(ps[j], ps[j + 1]), unpack2<T>(hw[j / 2]));
    lw[j / 2] = pack2<T>(lo.x, lo.y);
  }
  if constexpr (HC == 4) {
    const uint32_t off = tc::swz_offset<PRB>(jkey, cbase);
    *reinterpret_cast<uint2*>(hi_tile + off) = make_uint2(hw[0], hw[1]);
    *reinterpret_cast<uint2*>(lo_tile + off) = make_uint2(lw[0], lw[1]);
  } else {
#pragma unroll
    for (int c8 = 0; c8 < HC / 8; ++c8) {
      const uint32_t off = tc::swz_offset<PRB>(jkey, cbase + 8 * c8);
      *reinterpret_cast<uint4*>(hi_tile + off) = make_uint4(hw[4 * c8], hw[4 * c8 + 1], hw[4 * c8 + 2], hw[4 * c8 + 3]);
      *reinterpret_cast<uint4*>(lo_tile + off) = make_uint4(lw[4 * c8], lw[4 * c8 + 1], lw[4 * c8 + 2], lw[4 * c8 + 3]);
    }
  }
}

template <typename T, int D, int NPAD, int NS, int NPB, int ROUND>
__global__ void __launch_bounds__(NTH, 1)
    fused_scores_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                        const __grid_constant__ CUtensorMap qmap, TcArgs a) {
  using L = Lay<D, NPAD, NS, NPB>;
  constexpr bool BF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr int NREG = D / 64;            // 64-wide slabs of a K/V/Q/Y row
  constexpr int TMAX = L::TMAX;
  // 2*NPAD columns after the logit tiles: the y^T accumulator of pass 1, then S2
  // of pass 2 (hi part, lo part each)
  constexpr int S2COL = TMAX * NPAD;
  constexpr int HC = NPAD / 4;            // query columns per epilogue warp
  constexpr int PRB = L::PRB;
  static_assert(TMAX <= kMaxTiles, "s_done barriers");
  static_assert(HC >= 4 && HC <= 16, "column split");
  extern __shared__ uint8_t raw[];
  // the selection launched after this kernel may be scheduled as SMs free up; it
  // waits for this grid's completion before reading the scores
  pdl_launch_dependents();
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + L::BAR);
  uint64_t* freeb = full + NS;
  uint64_t* sdone = freeb + NS;
  uint64_t* bx = sdone + kMaxTiles;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + L::MISC);
  int* abort_flag = reinterpret_cast<int*>(sm + L::MISC + 8);
  float* mloc = reinterpret_cast<float*>(sm + L::MLOC);
  float* lse_s = reinterpret_cast<float*>(sm + L::LSE);
  float* yn_s = reinterpret_cast<float*>(sm + L::YN);
  int* bnd_s = reinterpret_cast<int*>(sm + L::BND);
  float* red = reinterpret_cast<float*>(sm + L::RED);
  float* xch = reinterpret_cast<float*>(sm + L::XCH);
  float* wts = reinterpret_cast<float*>(sm + L::WTS);
  float* vn_s = reinterpret_cast<float*>(sm + L::VN);
  float* sts = wts + kWts;

  const ScoreProblem& p = a.p;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int grp = blockIdx.x / a.gs, rank = blockIdx.x % a.gs;
  const int M = p.M, W = p.W, Lk = p.Lk;
  const int t0 = (int)(((long long)rank * a.tiles) / a.gs);
  const int nt = (int)(((long long)(rank + 1) * a.tiles) / a.gs) - t0;
  const int my_rounds = (grp < a.BH) ? min(a.rounds, (a.BH - grp + a.groups - 1) / a.groups) : 0;

  if (tid == 0) {
    for (int i = 0; i < L::NBAR; ++i) tc::mbar_init(&full[i], 1);
    // a ring slot is free after its MMA (commit) and kVnWarps arrivals: by the
    // epilogue warps that read a pass-1 V tile for ||v||^2, by the MMA thread
    // itself for K tiles and pass-2 V tiles
    for (int s = 0; s < NS; ++s) tc::mbar_init(&freeb[s], 1 + kVnWarps);
    tc::mbar_init(&bx[B_PREADY0], NEW);
    tc::mbar_init(&bx[B_PREADY1], NEW);
    tc::mbar_init(&bx[B_S2FREE0], NEW);
    tc::mbar_init(&bx[B_S2FREE1], NEW);
    tc::fence_mbar_init();
    *abort_flag = 0;
    if (blockIdx.x == 0) {
      a.trace[0] = gridDim.x;
      a.trace[1] = a.rounds;
      a.trace[2] = kTraceEv;
    }
  }
  if (warp == WARP_MMA) {
    tc::tmem_alloc(tslot, 512);
    tc::tmem_relinquish();
  }
  if (tid < NPAD) {
    bnd_s[tid] = (tid < M) ? (Lk - W + tid % W) : -1;
  }
  if (a.q_tma) {  // query rows M .. NPAD-1 of the Q operand stay zero (TMA writes rows < M)
    for (int i = tid; i < (NPAD - M) * D; i += NTH) {
      const int m = M + i / D, d = i % D;
      *reinterpret_cast<uint16_t*>(sm + L::QS + (d / 64) * L::RB + tc::sw128_offset(m, d % 64)) = 0;
    }
    tc::fence_proxy_async_smem();
  }
  if (tid == 0 && (grp & 1) && a.rounds >= kStaggerRounds) {  // the stagger: a timed wait, bounded by itself
    const uint64_t t_end = tc::globaltimer_ns() + (uint64_t)a.tmax_cta * kStaggerNsPerTile;
    while (tc::globaltimer_ns() < t_end) {
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tslot;

  volatile int* vabort = abort_flag;
  auto fail_wait = [&](int code) {
    *vabort = 1;
    atomicOr(a.status, code);
  };
  // bounded wait that also gives up as soon as another role aborted
  auto wait_bar = [&](uint64_t* b, uint32_t parity, int code) -> bool {
    if (*vabort) return false;
    if (tc::mbar_try_wait(b, parity)) return true;
    const uint64_t t_start = tc::globaltimer_ns();
    while (!tc::mbar_try_wait(b, parity)) {
      if (*vabort) return false;
      if (tc::globaltimer_ns() - t_start > a.wait_ns) {
        fail_wait(code);
        return false;
      }
    }
    return true;
  };

  if (warp == WARP_TMA) {
    // ======================= TMA producer =======================================
    // Load k: round k / (3 nt), stage (k / nt) % 3 (0: K pass 1, 1: V pass 1,
    // 2: V pass 2), tile k % nt.  V pass-1 loads keep their lines in L2 for pass 2.
    if (lane == 0) {
      const uint64_t pol_first = tc::policy_evict_first();
      const uint64_t pol_last = tc::policy_evict_last();
      tc::tma_prefetch_desc(&kmap);
      tc::tma_prefetch_desc(&vmap);
      // Q window of round r into the Q operand; QREADY's phase r completes on arrival
      auto load_q = [&](int r) {
        const int h = r * a.groups + grp;
        const int b = h / p.Hkv, hkv = h % p.Hkv;
        tc::mbar_arrive_expect_tx(&bx[B_QREADY], (uint32_t)(128 * M * NREG));
        for (int rr = 0; rr < NREG; ++rr)
          tc::tma_load_4d(sm + L::QS + rr * L::RB, &qmap, &bx[B_QREADY], 64 * rr, p.Lq - W, hkv * p.g, b);
      };
      if (a.q_tma) {
        tc::tma_prefetch_desc(&qmap);
        if (my_rounds > 0) load_q(0);
      }
      const uint32_t total = (uint32_t)my_rounds * 3u * (uint32_t)nt;
      uint32_t k = 0;
      for (; k < total; ++k) {
        const uint32_t slot = k % NS;
        if (a.q_tma && k % (3u * nt) == 2u * nt && (int)(k / (3u * nt)) + 1 < my_rounds) {
          // before this round's pass-2 loads: the round's logits are done with the
          // Q operand (its last logit tile has completed), so the next Q can come
          const int r = (int)(k / (3u * nt));
          if (!wait_bar(&sdone[nt - 1], r & 1, 5)) break;
          load_q(r + 1);
        }
        if (k >= NS && !wait_bar(&freeb[slot], ((k / NS) - 1) & 1, 2)) break;
        const int r = (int)(k / (3u * nt));
        const int stage = (int)((k / nt) % 3u);
        const int tile = (int)(k % nt);
        const int bh = r * a.groups + grp;
        tc::mbar_arrive_expect_tx(&full[slot], L::TILE);
        for (int rr = 0; rr < NREG; ++rr)
          tc::tma_load_4d_hint(sm + L::RING + slot * L::TILE + rr * 16384, stage == 0 ? &kmap : &vmap,
                               &full[slot], 64 * rr, (t0 + tile) * TK, bh % p.Hkv, bh / p.Hkv,
                               stage == 1 ? pol_last : pol_first);
      }
      // every issued copy has landed before the CTA may exit (already true unless
      // a wait gave up)
      for (uint32_t j = (k > (uint32_t)NS ? k - NS : 0u); j < k; ++j)
        if (!tc::mbar_wait(&full[j % NS], (j / NS) & 1, kWaitNs)) atomicOr(a.status, 3);
    }
  } else if (warp == WARP_MMA) {
    // ======================= MMA issuer ========================================
    if (lane == 0) {
      const uint32_t ring0 = tc::smem_addr(sm + L::RING);
      const uint32_t qs0 = tc::smem_addr(sm + L::QS);
      const uint32_t ps0 = tc::smem_addr(sm + L::PS);
      const uint32_t ys0 = tc::smem_addr(sm + L::YS);
      constexpr uint32_t ID_QK = tc::idesc_f16(BF16, 128, NPAD, false, false);
      // hi and lo halves stacked along N: one MMA per k-step reads the V tile once
      constexpr uint32_t ID_PV = tc::idesc_f16(BF16, 128, 2 * NPAD, true, true);
      // S2 = V [y_hi | y_lo]^T: the halves stacked along N (one MMA per k-step; the
      // tensor core's time here grows with the number of MMAs, not with N)
      constexpr uint32_t ID_S2 = tc::idesc_f16(BF16, 128, 2 * NPAD, false, false);
      constexpr uint32_t LBO_PV = (NREG == 2) ? 16384u : 0u;
      constexpr uint32_t LAYOUT_P = tc::layout_for_row_bytes(PRB);
      // descriptors of the Q and y operands; per k-step offsets are added to them
      const uint64_t qd0 = tc::smem_desc(qs0, 16, 1024);
      const uint64_t yd0 = tc::smem_desc(ys0, 16, 1024);
      uint32_t k = 0;  // ring position
      uint32_t c_pready[2] = {0, 0}, c_s2free[2] = {0, 0};
      for (int rd = 0; rd < my_rounds && !*vabort; ++rd) {
        if (!wait_bar(&bx[B_QREADY], rd & 1, 20)) break;
        tc::tc_fence_after();
        // pass 1a: S_i = K_i Q^T
        for (int i = 0; i < nt; ++i, ++k) {
          const uint32_t slot = k % NS;
          if (!wait_bar(&full[slot], (k / NS) & 1, 21)) break;
          tc::tc_fence_after();
          const uint64_t ad0 = tc::smem_desc(ring0 + slot * L::TILE, 16, 1024);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint64_t ad = tc::desc_add(ad0, (kk / 4) * 16384 + (kk % 4) * 32);
            const uint64_t bd = tc::desc_add(qd0, (kk / 4) * L::RB + (kk % 4) * 32);
            tc::mma_f16(tmem + i * NPAD, ad, bd, ID_QK, kk > 0);
          }
          tc::mma_commit(&freeb[slot]);
          tc::mbar_arrive_cnt(&freeb[slot], kVnWarps);
          tc::mma_commit(&sdone[i]);
        }
        // pass 1c: y^T += V_i^T (p_hi + p_lo)^T
        for (int i = 0; i < nt; ++i, ++k) {
          const uint32_t slot = k % NS;
          const int buf = i % NPB;
          if (!wait_bar(&full[slot], (k / NS) & 1, 22)) break;
          if (!wait_bar(&bx[B_PREADY0 + buf], c_pready[buf] & 1, 23)) break;
          ++c_pready[buf];
          tc::tc_fence_after();
          const uint64_t ad0 = tc::smem_desc(ring0 + slot * L::TILE, LBO_PV, 1024);
          const uint64_t bd0 = tc::smem_desc(ps0 + buf * 2 * L::PT, L::PT, 8 * PRB, LAYOUT_P);
          // B: the P_hi tile and, one leading-byte-offset (a tile) further, P_lo
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint64_t ad = tc::desc_add(ad0, kk * 2048);
            const uint64_t bd = tc::desc_add(bd0, kk * 16 * PRB);
            tc::mma_f16(tmem + S2COL, ad, bd, ID_PV, (i > 0 || kk > 0) ? 1u : 0u);
          }
          tc::mma_commit(&freeb[slot]);  // + the ||v||^2 warps' arrivals
          tc::mma_commit(&bx[B_PFREE0 + buf]);
        }
        tc::mma_commit(&bx[B_YDONE]);
        // pass 2: S2_i = V_i (y_hi + y_lo)^T
        if (!wait_bar(&bx[B_YREADY], rd & 1, 24)) break;
        tc::tc_fence_after();
        for (int i = 0; i < nt; ++i, ++k) {
          const uint32_t slot = k % NS;
          if (!wait_bar(&full[slot], (k / NS) & 1, 25)) break;
          if (i >= 1) {  // the epilogue has read S2 of tile i - 1
            if (!wait_bar(&bx[B_S2FREE0], c_s2free[0] & 1, 26)) break;
            ++c_s2free[0];
          }
          tc::tc_fence_after();
          const uint64_t ad0 = tc::smem_desc(ring0 + slot * L::TILE, 16, 1024);
          // B: the y_hi rows then the y_lo rows of each 64-wide slab (N = 2 * NPAD)
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint64_t ad = tc::desc_add(ad0, (kk / 4) * 16384 + (kk % 4) * 32);
            const uint64_t bd = tc::desc_add(yd0, (kk / 4) * 2 * L::RB + (kk % 4) * 32);
            tc::mma_f16(tmem + S2COL, ad, bd, ID_S2, kk > 0 ? 1u : 0u);
          }
          tc::mma_commit(&freeb[slot]);
          tc::mbar_arrive_cnt(&freeb[slot], kVnWarps);
          tc::mma_commit(&bx[B_S2READY0]);
        }
        // the last S2 is released after this round's epilogue read it (and every
        // logit tile of the round before it)
        if (nt > 0) {
          if (!wait_bar(&bx[B_S2FREE0], c_s2free[0] & 1, 27)) break;
          ++c_s2free[0];
        }
      }
      tc::mma_commit(&bx[B_FIN]);
      if (!tc::mbar_wait(&bx[B_FIN], 0, kWaitNs)) atomicOr(a.status, 28);
    }
  } else {
    // ======================= epilogue: warps 0-15 =============================
    const int q = warp & 3;              // TMEM lane quadrant: keys 32q .. 32q+31 of a tile
    const int cg = warp >> 2;            // query-column group
    const int et = tid;                  // 0 .. NEPI-1
    const int jkey = q * 32 + lane;      // key within a tile
    const uint32_t lrow = (uint32_t)(q * 32) << 16;
    const int cbase = cg * HC;
    uint32_t c_pfree[2] = {0, 0}, c_s2r[2] = {0, 0};
    const bool stamper = (et == 0);
    auto stamp = [&](int rd, int ev) {
      if (stamper) a.trace[3 + ((size_t)blockIdx.x * a.rounds + rd) * kTraceEv + ev] = tc::globaltimer_ns();
    };
    // which of my columns are real query rows
    // (column j of this warp is a real query row when cbase + j < M)
    // every column of this warp is a real query row: tiles below the causal edge
    // then need no per-pair masks (the fast loops below)
    const bool allcols = cbase + HC <= M;

    for (int rd = 0; rd < my_rounds; ++rd) {
      const int h = rd * a.groups + grp;
      const int b = h / p.Hkv, hkv = h % p.Hkv;
      stamp(rd, TR_START);

      // ---- Q window -> SW128 K-major operand (unless the TMA warp loads it) ------
      if (!a.q_tma) {
        const T* qp = reinterpret_cast<const T*>(p.q);
#pragma unroll 4
        for (int i = et; i < NPAD * D; i += NEPI) {
          const int m = i / D, d = i % D;
          uint16_t v = 0;
          if (m < M) {
            const int qh = hkv * p.g + m / W;
            const int qpos = p.Lq - W + m % W;
            const T x = qp[(int64_t)b * p.q_sb + (int64_t)qh * p.q_sh + (int64_t)qpos * p.q_ss + (int64_t)d * p.q_sd];
            v = *reinterpret_cast<const uint16_t*>(&x);
          }
          *reinterpret_cast<uint16_t*>(sm + L::QS + (d / 64) * L::RB + tc::sw128_offset(m, d % 64)) = v;
        }
        tc::fence_proxy_async_smem();
        tc::tc_fence_before();
        epi_sync();
        if (et == 0) tc::mbar_arrive(&bx[B_QREADY]);
      }

      // ---- pass 1b: local max per query row, as logit tiles complete ----------
      float mx[HC];
#pragma unroll
      for (int j = 0; j < HC; ++j) mx[j] = -INFINITY;
      for (int i = 0; i < nt; ++i) {
        wait_bar(&sdone[i], rd & 1, 30);
        tc::tc_fence_after();
        float s[HC];
        tmem_ld<HC>(tmem + lrow + i * NPAD + cbase, s);
        const int key = (t0 + i) * TK + jkey;
        const bool edge = (t0 + i) * TK + TK - 1 > Lk - W;
        // max of the raw logits; scaled by c > 0 after the loop (rounding is
        // monotonic, so max(l) * c is the max of the rounded l * c)
        if (!edge && allcols) {
#pragma unroll
          for (int j = 0; j < HC; ++j) mx[j] = fmaxf(mx[j], s[j]);
        } else {
#pragma unroll
          for (int j = 0; j < HC; ++j) {
            const bool ok = edge ? (key <= bnd_s[cbase + j] && key < Lk) : (cbase + j < M);
            mx[j] = fmaxf(mx[j], ok ? s[j] : -INFINITY);
          }
        }
      }
#pragma unroll
      for (int j = 0; j < HC; ++j) mx[j] *= a.c;
      stamp(rd, TR_LOGITS);
      {
        const float col = col_reduce<HC, true>(mx, lane);
        if (lane < HC) red[q * NPAD + cbase + lane] = col;
      }
      epi_sync();
      if (et < NPAD) {
        float m4 = red[et];
#pragma unroll
        for (int w = 1; w < 4; ++w) m4 = fmaxf(m4, red[w * NPAD + et]);
        mloc[et] = m4;
      }
      epi_sync();
      stamp(rd, TR_MAX);

      // ---- pass 1c: p = exp2(l - m) -> hi/lo P tiles -----------------------------
      float ssum[HC];
#pragma unroll
      for (int j = 0; j < HC; ++j) ssum[j] = 0.f;
      float nml[HC];  // minus the row maxima
#pragma unroll
      for (int j = 0; j < HC; ++j) nml[j] = -mloc[cbase + j];
      for (int i = 0; i < nt; ++i) {
        const int buf = i % NPB;
        if (i >= NPB) {
          wait_bar(&bx[B_PFREE0 + buf], c_pfree[buf] & 1, 31);
          ++c_pfree[buf];
        }
        float s[HC];
        tc::tc_fence_after();
        tmem_ld<HC>(tmem + lrow + i * NPAD + cbase, s);
        const int key = (t0 + i) * TK + jkey;
        const bool edge = (t0 + i) * TK + TK - 1 > Lk - W;
        float ps[HC];
        if (!edge && allcols) {
          // every pair is a valid (key, query row) and the row maxima are finite
#pragma unroll
          for (int j = 0; j < HC; j += 2) {
            const float2 x = f2_fma(make_float2(s[j], s[j + 1]), make_float2(a.c, a.c),
                                    make_float2(nml[j], nml[j + 1]));
            const float2 pr = make_float2(ex2f(x.x), ex2f(x.y));
            const float2 sm2 = f2_add(make_float2(ssum[j], ssum[j + 1]), pr);
            ssum[j] = sm2.x;
            ssum[j + 1] = sm2.y;
            const float2 sc = BF16 ? pr : f2_mul(pr, make_float2(a.pscale, a.pscale));
            ps[j] = sc.x;
            ps[j + 1] = sc.y;
          }
        } else {
#pragma unroll
          for (int j = 0; j < HC; j += 2) {
            const bool ok0 = (edge ? (key <= bnd_s[cbase + j] && key < Lk) : (cbase + j < M)) && nml[j] != INFINITY;
            const bool ok1 =
                (edge ? (key <= bnd_s[cbase + j + 1] && key < Lk) : (cbase + j + 1 < M)) && nml[j + 1] != INFINITY;
            const float2 x = f2_fma(make_float2(s[j], s[j + 1]), make_float2(a.c, a.c),
                                    make_float2(nml[j], nml[j + 1]));
            const float2 pr = make_float2(ok0 ? ex2f(x.x) : 0.f, ok1 ? ex2f(x.y) : 0.f);
            const float2 sm2 = f2_add(make_float2(ssum[j], ssum[j + 1]), pr);
            ssum[j] = sm2.x;
            ssum[j + 1] = sm2.y;
            const float2 sc = f2_mul(pr, make_float2(a.pscale, a.pscale));
            ps[j] = sc.x;
            ps[j + 1] = sc.y;
          }
        }
        uint8_t* pb = sm + L::PS + buf * 2 * L::PT;
        store_p<T, HC, PRB>(pb, pb + L::PT, jkey, cbase, ps);
        tc::fence_proxy_async_smem();
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&bx[B_PREADY0 + buf]);
        // ||v_j||^2 of V tile i, by column group i % 4; the tile's ring slot waits
        // for these four warps.  Its full phase is unambiguous: the slot's previous
        // load was consumed before this round's logits (K) or P.V (tile i - NS).
        if (cg == (i & 3)) {
          const uint32_t kpos = (uint32_t)rd * 3u * nt + (uint32_t)nt + (uint32_t)i;  // ring position
          const uint32_t slot = kpos % NS;
          wait_bar(&full[slot], (kpos / NS) & 1, 32);
          float2 vn2 = make_float2(0.f, 0.f);
#pragma unroll
          for (int rr = 0; rr < NREG; ++rr) {
            const uint8_t* vt = sm + L::RING + slot * L::TILE + rr * 16384 + jkey * 128;
#pragma unroll
            for (int c8 = 0; c8 < 8; ++c8) {
              const uint4 r4 = *reinterpret_cast<const uint4*>(vt + ((c8 ^ (jkey & 7)) << 4));
              const uint32_t w4[4] = {r4.x, r4.y, r4.z, r4.w};
#pragma unroll
              for (int k2 = 0; k2 < 4; ++k2) {
                const float2 x = unpack2<T>(w4[k2]);
                vn2 = f2_fma(x, x, vn2);
              }
            }
          }
          vn_s[i * TK + jkey] = vn2.x + vn2.y;
          __syncwarp();
          if (lane == 0) tc::mbar_arrive(&freeb[slot]);
        }
      }
      // y^T complete
      if (nt > 0) wait_bar(&bx[B_YDONE], rd & 1, 33);
      // the P buffers of the last tiles were released by that too
      for (int i = (nt >= NPB ? nt - NPB : 0); i < nt; ++i) {
        const int buf = i % NPB;
        wait_bar(&bx[B_PFREE0 + buf], c_pfree[buf] & 1, 34);
        ++c_pfree[buf];
      }
      tc::tc_fence_after();
      stamp(rd, TR_PV);

      // ---- partial (m, s, y) of this CTA -----------------------------------------
      {
        const float col = col_reduce<HC, false>(ssum, lane);
        if (lane < HC) red[q * NPAD + cbase + lane] = col;
      }
      epi_sync();
      const size_t prow = ((size_t)h * a.gs + rank) * M;
      if (et < M) {
        const float s4 = red[et] + red[NPAD + et] + red[2 * NPAD + et] + red[3 * NPAD + et];
        __stcg(a.part_m + prow + et, mloc[et]);
        __stcg(a.part_s + prow + et, s4);
      }
      {
        const float inv = 1.0f / a.pscale;
        const int d = q * 32 + lane;  // TMEM lane of the y^T accumulator = d
        if (d < D) {
          float v[HC], vl[HC];
          if (nt > 0) {
            tmem_ld<HC>(tmem + lrow + S2COL + cbase, v);
            tmem_ld<HC>(tmem + lrow + S2COL + NPAD + cbase, vl);
          }
#pragma unroll
          for (int j = 0; j < HC; ++j)
            if (cbase + j < M) __stcg(a.part_y + (prow + cbase + j) * D + d, nt > 0 ? (v[j] + vl[j]) * inv : 0.f);
        }
      }
      tc::tc_fence_before();

      // ---- group barrier A, distributed merge, group barrier B --------------------
      auto group_barrier = [&](int* ctr) {
        epi_sync();
        if (et == 0 && !*vabort) {
          // release: the epilogue's stores before the named barrier (partials,
          // merged y) are visible to every CTA that acquires the count
          asm volatile("red.release.gpu.global.add.s32 [%0], 1;" ::"l"(ctr) : "memory");
          const uint64_t t_start = tc::globaltimer_ns();
          while (true) {
            int v;
            asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(ctr) : "memory");
            if (v >= a.gs) break;
            if (*vabort) break;
            if (tc::globaltimer_ns() - t_start > a.wait_ns) { fail_wait(35); break; }
          }
        }
        epi_sync();  // orders the other threads' loads after the acquire
      };
      group_barrier(a.ctr + 2 * h);
      stamp(rd, TR_BAR_A);
      {
        // This CTA merges elements [e0, e1) of the head's M x D y with the
        // max-rescale rule (dropkv_triton.py:441-452), in a fixed order. The
        // slices start on multiples of 4 elements (E = M D is one), so the
        // partials are read as 16-byte vectors.
        const int E = M * D;
        const int e0 = (int)((((long long)rank * E) / a.gs) & ~3LL);
        const int e1 = (int)((((long long)(rank + 1) * E) / a.gs) & ~3LL);
        const int ne = e1 - e0;
        const size_t hb = (size_t)h * a.gs;
        float* acc = reinterpret_cast<float*>(sm + L::PS);  // P tiles are idle here
        constexpr int CAP = NPB * 2 * L::PT / 4;            // floats
        if (ne > 0) {
          const int m_lo = e0 / D, nrow = (e1 - 1) / D - m_lo + 1;
          const int nst = nrow * a.gs;
          // weighted sums in chunks of elements whose partials fit the P tiles; the
          // first chunk's loads go out together with the rows' partial maxima and
          // sums (one L2 round trip for the whole slice when it fits one chunk)
          const int ec = max(4, min(ne, (CAP / a.gs) & ~3));  // a multiple of 4, as ne is
          for (int cs = 0; cs < ne; cs += ec) {
            const int cn = min(ec, ne - cs);
            // the rows' partial maxima and sums (first chunk only): 2 nst values,
            // nst = nrow gs <= M + 2 gs, so two per thread cover the plans of a
            // 148-SM GPU (M <= 64); a loop takes any rest
            const int nms = cs == 0 ? 2 * nst : 0;
            float msv[2];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const int k = et + u * NEPI;
              msv[u] = 0.f;
              if (k < nms) {
                const int kk = k < nst ? k : k - nst;
                const int r = kk / a.gs, c = kk - r * a.gs;
                msv[u] = __ldcg((k < nst ? a.part_m : a.part_s) + (hb + c) * M + m_lo + r);
              }
            }
            // vector k = c cn4 + e (partial c, elements 4e .. 4e + 3 of the chunk),
            // stepped by NEPI without divisions; it lands at acc[4k] = acc[c cn + 4e]
            const int cn4 = cn / 4, npairs4 = a.gs * cn4;
            const int dq = NEPI / cn4, dr = NEPI - dq * cn4;
            int c = et / cn4, e = et - (et / cn4) * cn4;
            for (int k0 = 0; k0 < npairs4; k0 += 4 * NEPI) {
              float4 val[4];
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                val[u] = c < a.gs ? __ldcg(reinterpret_cast<const float4*>(a.part_y + (hb + c) * E + e0 + cs) + e)
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
                c += dq;
                e += dr;
                if (e >= cn4) {
                  e -= cn4;
                  ++c;
                }
              }
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                const int k = k0 + u * NEPI + et;
                if (k < npairs4) reinterpret_cast<float4*>(acc)[k] = val[u];
              }
            }
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const int k = et + u * NEPI;
              if (k < nst) wts[k] = msv[u];
              else if (k < nms) sts[k - nst] = msv[u];
            }
            for (int k = et + 2 * NEPI; k < nms; k += NEPI) {
              const int kk = k < nst ? k : k - nst;
              const int r = kk / a.gs, c = kk - r * a.gs;
              const float x = __ldcg((k < nst ? a.part_m : a.part_s) + (hb + c) * M + m_lo + r);
              if (k < nst) wts[k] = x;
              else sts[k - nst] = x;
            }
            epi_sync();
            if (cs == 0) {  // the rows' maxima and the weights of the partials
              for (int r = warp; r < nrow; r += NEW) {
                float mxr = -INFINITY;
                for (int c = lane; c < a.gs; c += 32) mxr = fmaxf(mxr, wts[r * a.gs + c]);
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) mxr = fmaxf(mxr, __shfl_xor_sync(0xffffffffu, mxr, o));
                float tot = 0.f;
                for (int c = lane; c < a.gs; c += 32) {
                  const float pm = wts[r * a.gs + c];
                  const float w = (pm == -INFINITY) ? 0.f : exp2f(pm - mxr);
                  wts[r * a.gs + c] = w;
                  tot = fmaf(w, sts[r * a.gs + c], tot);
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
                if (lane == 0) {
                  red[r] = tot;
                  red[NPAD + r] = mxr;
                }
              }
              epi_sync();
            }
            // SPL threads per element, each over a fixed subset of the partials
            const int spl = max(1, min(8, NEPI / cn));
            for (int idx = et; idx < cn * spl; idx += NEPI) {
              const int e = idx / spl, sp = idx % spl;
              const int eg = e0 + cs + e, m = eg / D;
              const float* wr = wts + (m - m_lo) * a.gs;
              float sacc = 0.f;
              for (int c = sp; c < a.gs; c += spl) sacc = fmaf(wr[c], acc[c * cn + e], sacc);
              if (spl == 1) __stcg(a.y_g + (size_t)h * E + eg, sacc / red[m - m_lo]);
              else xch[idx] = sacc;
            }
            if (spl > 1) {
              epi_sync();
              for (int e = et; e < cn; e += NEPI) {
                float sacc = 0.f;
                for (int sp = 0; sp < spl; ++sp) sacc += xch[e * spl + sp];
                const int eg = e0 + cs + e, m = eg / D;
                __stcg(a.y_g + (size_t)h * E + eg, sacc / red[m - m_lo]);
              }
            }
            epi_sync();  // acc and xch are refilled by the next chunk
          }
          if (et < nrow && e0 <= (m_lo + et) * D)
            __stcg(a.lse_g + (size_t)h * M + m_lo + et, red[NPAD + et] + log2f(red[et]));
        }
      }
      stamp(rd, TR_MERGE);
      group_barrier(a.ctr + 2 * h + 1);
      stamp(rd, TR_BAR_B);

      // ---- y (hi/lo) -> shared memory; lse, ||y||^2 --------------------------------
      {
        constexpr int TPRY = (NEPI / NPAD < D / 8) ? NEPI / NPAD : D / 8;  // threads per row
        constexpr int DPT = D / TPRY;
        const int m = et / TPRY, dbase = (et % TPRY) * DPT;
        float n2 = 0.f;
        if (m < NPAD) {
#pragma unroll
          for (int d8 = 0; d8 < DPT; d8 += 8) {
            const int d = dbase + d8;
            float y[8];
            if (m < M) {
              const float4 u0 = __ldcg(reinterpret_cast<const float4*>(a.y_g + ((size_t)h * M + m) * D + d));
              const float4 u1 = __ldcg(reinterpret_cast<const float4*>(a.y_g + ((size_t)h * M + m) * D + d + 4));
              y[0] = u0.x; y[1] = u0.y; y[2] = u0.z; y[3] = u0.w;
              y[4] = u1.x; y[5] = u1.y; y[6] = u1.z; y[7] = u1.w;
            } else {
#pragma unroll
              for (int k2 = 0; k2 < 8; ++k2) y[k2] = 0.f;
            }
            uint32_t hw[4], lw[4];
#pragma unroll
            for (int k2 = 0; k2 < 8; k2 += 2) {
              n2 = fmaf(y[k2], y[k2], n2);
              n2 = fmaf(y[k2 + 1], y[k2 + 1], n2);
              hw[k2 / 2] = pack2<T>(y[k2], y[k2 + 1]);
              const float2 back = unpack2<T>(hw[k2 / 2]);
              lw[k2 / 2] = pack2<T>(y[k2] - back.x, y[k2 + 1] - back.y);
            }
            const uint32_t off = (d / 64) * 2 * L::RB + m * 128 + ((((d % 64) >> 3) ^ (m & 7)) << 4);
            *reinterpret_cast<uint4*>(sm + L::YS + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
            *reinterpret_cast<uint4*>(sm + L::YS + L::RB + off) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
          }
        }
#pragma unroll
        for (int o = 1; o < TPRY; o <<= 1) n2 += __shfl_xor_sync(0xffffffffu, n2, o);
        if (m < NPAD && et % TPRY == 0) {
          yn_s[m] = n2;
          lse_s[m] = (m < M) ? __ldcg(a.lse_g + (size_t)h * M + m) : 0.f;
        }
      }
      tc::fence_proxy_async_smem();
      tc::tc_fence_before();
      epi_sync();
      if (et == 0) tc::mbar_arrive(&bx[B_YREADY]);
      stamp(rd, TR_YSTAGE);

      // ---- pass 2: score epilogue over S (TMEM, pass 1), S2 = <v, y> and ||v||^2 (pass 1c) ----
      float nlse[HC], ynl[HC];
#pragma unroll
      for (int j = 0; j < HC; ++j) {
        nlse[j] = -lse_s[cbase + j];
        ynl[j] = yn_s[cbase + j];
      }
      for (int i = 0; i < nt; ++i) {
        const int buf = i & 1;  // exchange buffer
        wait_bar(&bx[B_S2READY0], c_s2r[0] & 1, 36);
        ++c_s2r[0];
        tc::tc_fence_after();
        float s[HC], s2[HC], s2l[HC];
        tmem_ld<HC>(tmem + lrow + i * NPAD + cbase, s);
        tmem_ld<HC>(tmem + lrow + S2COL + cbase, s2);
        tmem_ld<HC>(tmem + lrow + S2COL + NPAD + cbase, s2l);
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&bx[B_S2FREE0]);
#pragma unroll
        for (int j = 0; j < HC; j += 2) {  // <v, y> = <v, y_hi> + <v, y_lo>
          const float2 t = f2_add(make_float2(s2[j], s2[j + 1]), make_float2(s2l[j], s2l[j + 1]));
          s2[j] = t.x;
          s2[j + 1] = t.y;
        }
        const int key = (t0 + i) * TK + jkey;
        const bool edge = (t0 + i) * TK + TK - 1 > Lk - W;
        // pairs of query columns: w = (p / (1 - p + eps))^2 with p rounded to the
        // input dtype; sums of w, w <v, y> and w ||y||^2 over this thread's columns
        float2 sw2 = make_float2(0.f, 0.f), sb2 = sw2, sc2 = sw2;
        if (!edge && allcols) {
#pragma unroll
          for (int j = 0; j < HC; j += 2) {
            const float2 x = f2_fma(make_float2(s[j], s[j + 1]), make_float2(a.c, a.c),
                                    make_float2(nlse[j], nlse[j + 1]));
            // p = 2^x <= 1 up to the rounding of x (a few ulps above 1 at most),
            // which rounding p to bf16 / fp16 maps to 1: the clamp is needed only
            // when p keeps fp32
            const float2 pr = ROUND == DROPKV_ROUND_NONE
                                  ? make_float2(fminf(ex2f(x.x), 1.f), fminf(ex2f(x.y), 1.f))
                                  : round_p2<ROUND>(make_float2(ex2f(x.x), ex2f(x.y)));
            const float2 den = f2_add(f2_sub(make_float2(1.f, 1.f), pr), make_float2(p.eps, p.eps));
            const float2 ratio = f2_mul(pr, make_float2(rcpf(den.x), rcpf(den.y)));
            const float2 w = f2_mul(ratio, ratio);
            sw2 = f2_add(sw2, w);
            sb2 = f2_fma(w, make_float2(s2[j], s2[j + 1]), sb2);
            sc2 = f2_fma(w, make_float2(ynl[j], ynl[j + 1]), sc2);
          }
        } else {
#pragma unroll
          for (int j = 0; j < HC; j += 2) {
            const bool ok0 = edge ? (key <= bnd_s[cbase + j] && key < Lk) : (cbase + j < M);
            const bool ok1 = edge ? (key <= bnd_s[cbase + j + 1] && key < Lk) : (cbase + j + 1 < M);
            const float2 x = f2_fma(make_float2(s[j], s[j + 1]), make_float2(a.c, a.c),
                                    make_float2(nlse[j], nlse[j + 1]));
            const float2 pr = round_p2<ROUND>(make_float2(fminf(ex2f(x.x), 1.f), fminf(ex2f(x.y), 1.f)));
            const float2 den = f2_add(f2_sub(make_float2(1.f, 1.f), pr), make_float2(p.eps, p.eps));
            const float2 ratio = f2_mul(pr, make_float2(rcpf(den.x), rcpf(den.y)));
            float2 w = f2_mul(ratio, ratio);
            w.x = ok0 ? w.x : 0.f;
            w.y = ok1 ? w.y : 0.f;
            sw2 = f2_add(sw2, w);
            sb2 = f2_fma(w, make_float2(s2[j], s2[j + 1]), sb2);
            sc2 = f2_fma(w, make_float2(ynl[j], ynl[j + 1]), sc2);
          }
        }
        float sw = sw2.x + sw2.y, sb = sb2.x + sb2.y, sc = sc2.x + sc2.y;
        // column groups 1-3 hand their sums to group 0 (fixed order: deterministic)
        float* xb = xch + buf * 9 * TK;
        if (cg > 0) {
          float* xg = xb + (cg - 1) * 3 * TK;
          xg[jkey] = sw;
          xg[TK + jkey] = sb;
          xg[2 * TK + jkey] = sc;
        }
        quad_sync(q);
        if (cg == 0 && key < Lk) {
#pragma unroll
          for (int g3 = 0; g3 < 3; ++g3) {
            const float* xg = xb + g3 * 3 * TK;
            sw += xg[jkey];
            sb += xg[TK + jkey];
            sc += xg[2 * TK + jkey];
          }
          const float vn = vn_s[i * TK + jkey];
          p.scores[(size_t)h * Lk + key] = (sw * vn - 2.f * sb + sc) / (float)p.g;
        }
      }
      stamp(rd, TR_PASS2);
    }
  }

  // ---- teardown: every MMA finished (MMA lane waited on B_FIN), TMEM released --
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  if (warp == WARP_MMA) tc::tmem_dealloc(tmem, 512);
}

}  // namespace

// ---------------------------------------------------------------------------
// Host planning and launch
// ---------------------------------------------------------------------------
// Test hooks (process-wide): the limit of the scorer's waits on other roles and
// CTAs, and a switch that makes the first group barrier of every launch
// unreachable, so that a test can drive the timeout path on a GPU without any
// fault: the waits give up, the kernel records a status and ends.
static std::atomic<uint64_t> g_wait_ns{kWaitNs};
static std::atomic<int> g_block_barrier{0};

void tc_test_set_wait_ns(uint64_t ns) { g_wait_ns.store(ns ? ns : kWaitNs); }
void tc_test_block_barrier(int on) { g_block_barrier.store(on ? 1 : 0); }

struct TcPlan {
  bool ok;
  int npad, tmax, tiles, gs, groups, rounds, nctas;
  size_t off_ctr, off_status, off_trace, off_pm, off_ps, off_py, off_y, off_lse, bytes;
};

static int tc_npad(int M) { return M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : 0; }

static TcPlan plan_tc_compute(int BH, int Lk, int M, int D, int nsm) {
  TcPlan t;
  std::memset(&t, 0, sizeof(t));
  t.npad = tc_npad(M);
  if (!t.npad || (D != 64 && D != 128)) return t;
  t.tmax = (512 - 2 * t.npad) / t.npad;
  t.tiles = (Lk + TK - 1) / TK;
  const int gs_min = (t.tiles + t.tmax - 1) / t.tmax;
  if (gs_min > nsm) return t;
  double best = 1e30;
  for (int gs = gs_min; gs <= std::min(t.tiles, nsm); ++gs) {
    int groups = std::min(nsm / gs, BH);
    int rounds = (BH + groups - 1) / groups;
    int per = (t.tiles + gs - 1) / gs;
    double cost = rounds * (per + 3.0);  // ~3 tile-times of barrier/merge per round
    if (cost < best - 1e-9) {
      best = cost;
      t.gs = gs;
      t.groups = groups;
      t.rounds = rounds;
    }
  }
  if (t.gs > kMaxGs) return t;
  t.nctas = t.gs * t.groups;
  size_t off = 0;
  t.off_ctr = off; off = align_up(off + (size_t)2 * BH * 4, 256);
  t.off_status = off; off = align_up(off + 4, 256);
  t.off_trace = off; off = align_up(off + 8 * (3 + (size_t)t.nctas * t.rounds * kTraceEv), 256);
  t.off_pm = off; off = align_up(off + (size_t)BH * t.gs * M * 4, 256);
  t.off_ps = off; off = align_up(off + (size_t)BH * t.gs * M * 4, 256);
  t.off_py = off; off = align_up(off + (size_t)BH * t.gs * M * D * 4, 256);
  t.off_y = off; off = align_up(off + (size_t)BH * M * D * 4, 256);
  t.off_lse = off; off = align_up(off + (size_t)BH * M * 4, 256);
  t.bytes = off;
  t.ok = true;
  return t;
}

// The plan of a problem is asked for several times per call (workspace size,
// scorer choice, launch); the last 16 distinct problems are kept.
TcPlan plan_tc(int BH, int Lk, int M, int D, int nsm) {
  struct Entry {
    int BH, Lk, M, D, nsm;
    TcPlan t;
  };
  static std::mutex mu;
  static Entry cache[16] = {};
  static int next = 0;
  {
    std::lock_guard<std::mutex> lock(mu);
    for (const Entry& e : cache)
      if (e.BH == BH && e.Lk == Lk && e.M == M && e.D == D && e.nsm == nsm) return e.t;
  }
  const TcPlan t = plan_tc_compute(BH, Lk, M, D, nsm);
  std::lock_guard<std::mutex> lock(mu);
  cache[next] = Entry{BH, Lk, M, D, nsm, t};
  next = (next + 1) % 16;
  return t;
}

template <typename T, int D, int NPAD, int ROUND>
static int launch_fused_t(const ScoreProblem& p, const TcPlan& t, void* ws, cudaStream_t st) {
  // ring depth and P double-buffering as far as 227 KB of shared memory allows
  constexpr int NS = (D == 128) ? (NPAD == 16 ? 5 : NPAD == 32 ? 4 : 3) : 8;
  constexpr int NPB = (NPAD == 64) ? 1 : 2;
  using L = Lay<D, NPAD, NS, NPB>;
  static_assert(L::ALLOC <= 232448, "shared memory budget");
  CUtensorMap km, vm;
  const bool bf16 = std::is_same<T, __nv_bfloat16>::value;
  const int BH = p.B * p.Hkv;
  int rc = make_kv_tensor_map_4d(&km, p.k, p.B, p.Hkv, p.Lk, D, bf16, p.kv_sb, p.kv_sh, p.kv_ss);
  if (rc) return rc;
  rc = make_kv_tensor_map_4d(&vm, p.v, p.B, p.Hkv, p.Lk, D, bf16, p.kv_sb, p.kv_sh, p.kv_ss);
  if (rc) return rc;
  CUtensorMap qm;
  std::memset(&qm, 0, sizeof(qm));
  const bool q_tma = make_q_tensor_map(&qm, p, bf16);
  char* base = reinterpret_cast<char*>(ws);
  TcArgs a;
  a.p = p;
  a.BH = BH;
  a.gs = t.gs; a.groups = t.groups; a.rounds = t.rounds; a.tiles = t.tiles; a.tmax = t.tmax;
  a.tmax_cta = (t.tiles + t.gs - 1) / t.gs;
  a.c = (float)(1.4426950408889634 / std::sqrt((double)p.D));
  a.pscale = bf16 ? 1.0f : 32768.0f;
  a.q_tma = q_tma ? 1 : 0;
  a.ctr = reinterpret_cast<int*>(base + t.off_ctr);
  a.status = p.status ? p.status : reinterpret_cast<int*>(base + t.off_status);
  a.trace = reinterpret_cast<unsigned long long*>(base + t.off_trace);
  a.part_m = reinterpret_cast<float*>(base + t.off_pm);
  a.part_s = reinterpret_cast<float*>(base + t.off_ps);
  a.part_y = reinterpret_cast<float*>(base + t.off_py);
  a.y_g = reinterpret_cast<float*>(base + t.off_y);
  a.lse_g = reinterpret_cast<float*>(base + t.off_lse);
  a.wait_ns = g_wait_ns.load();
  if (cudaMemsetAsync(base + t.off_ctr, 0, t.off_pm - t.off_ctr, st) != cudaSuccess)
    return fail(DROPKV_ERR_CUDA, "memset of barrier counters failed");
  // test hook: head 0's first group-barrier counter starts negative (0x80808080),
  // so the arrivals of its CTAs never reach the group size
  if (g_block_barrier.load() && cudaMemsetAsync(base + t.off_ctr, 0x80, 4, st) != cudaSuccess)
    return fail(DROPKV_ERR_CUDA, "memset of the blocked barrier counter failed");
  auto kern = fused_scores_kernel<T, D, NPAD, NS, NPB, ROUND>;
  static DeviceOnce attr_done;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_done.done(dev)) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::ALLOC) != cudaSuccess)
      return fail(DROPKV_ERR_CUDA, "cannot set shared memory size %d", L::ALLOC);
    attr_done.mark(dev);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(t.nctas);
  cfg.blockDim = dim3(NTH);
  cfg.dynamicSmemBytes = L::ALLOC;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, km, vm, qm, a);
  if (e != cudaSuccess) return fail(DROPKV_ERR_CUDA, "fused scorer launch: %s", cudaGetErrorString(e));
  return check_launch("fused_scores", 2);
}

bool tc_supported(int dtype, int M, int D, int BH, int Lk) {
  if (dtype != DROPKV_DTYPE_BF16 && dtype != DROPKV_DTYPE_F16) return false;
  TcPlan t = plan_tc(BH, Lk, M, D, num_sms_current_device());
  return t.ok;
}

size_t tc_workspace_bytes(int M, int D, int BH, int Lk) {
  TcPlan t = plan_tc(BH, Lk, M, D, num_sms_current_device());
  return t.ok ? t.bytes : 0;
}

size_t tc_status_offset(int M, int D, int BH, int Lk) {
  TcPlan t = plan_tc(BH, Lk, M, D, num_sms_current_device());
  return t.off_status;
}

int launch_scores_tc(const ScoreProblem& p, int dtype, void* ws, cudaStream_t st) {
  const int BH = p.B * p.Hkv;
  TcPlan t = plan_tc(BH, p.Lk, p.M, p.D, num_sms_current_device());
  if (!t.ok) return fail(DROPKV_ERR_UNSUPPORTED, "tensor-core scorer does not cover this shape");
  const bool bf = dtype == DROPKV_DTYPE_BF16;
  const bool rnd = p.round_mode != DROPKV_ROUND_NONE;
#define DKV_CASE(TT, DD, NN, RR)                      \
  if (p.D == DD && t.npad == NN && rnd == (RR != 0)) \
    return launch_fused_t<TT, DD, NN, RR>(p, t, ws, st);
#define DKV_SHAPES(TT, RR) \
  DKV_CASE(TT, 128, 16, RR) DKV_CASE(TT, 128, 32, RR) DKV_CASE(TT, 128, 64, RR) \
  DKV_CASE(TT, 64, 16, RR) DKV_CASE(TT, 64, 32, RR) DKV_CASE(TT, 64, 64, RR)
  if (bf) {
    DKV_SHAPES(__nv_bfloat16, 0)
    DKV_SHAPES(__nv_bfloat16, DROPKV_ROUND_BF16)
  } else {
    DKV_SHAPES(__half, 0)
    DKV_SHAPES(__half, DROPKV_ROUND_F16)
  }
#undef DKV_SHAPES
#undef DKV_CASE
  return fail(DROPKV_ERR_UNSUPPORTED, "no tensor-core kernel for D=%d, M=%d", p.D, p.M);
}

}  // namespace dropkv
