// ozaki.cuh — the exact path's GEMMs on the int8 tensor cores, with the
// same f32 results as the FP64 kernel (k_dgemm_exact).
//
// matmulOracle (forward/oracle.ts:114-125) stores f32(c) where c is one f64
// chain over k in order: c_k = fl(c_(k-1) + a_k·b_k), the products exact (two
// f32 factors). That chain differs from the exact dot product y = Σ a_k b_k by
// at most γ_(K-1)·Σ|a_k b_k| (γ_n = n·u / (1 − n·u), u = 2^-53). So whenever
// y is known to lie in an interval [ŷ − E, ŷ + E] that also holds the chain
// and whose two ends round to the same f32, that f32 IS the oracle's stored
// value (rounding is monotone). The few outputs whose interval straddles a
// rounding boundary are listed and recomputed by the sequential chain
// (k_oz_fixup), so every output equals the FP64 kernel's bit for bit.
//
// ŷ comes from the integer tensor cores (the slicing idea of Ozaki, Ogita &
// Oishi, "Error-free transformations of matrix multiplication by using fast
// routines of matrix multiplication and its applications", Numer. Algorithms
// 59, 2012, in the integer form of Ootomo, Ozaki & Yokota, IJHPCA 2024):
//
//   each row x of A (and of B, the weights [N, K]) gets an exponent e with
//   max|x| < 2^e and six slices of x' = x·2^-e ∈ (−1, 1):
//     s0 = floor(x'·2^7) ∈ [−128, 127] (signed int8), r0 = x'·2^7 − s0 ∈ [0, 1),
//     s_i = floor(r_(i−1)·2^8) ∈ [0, 255] (unsigned int8), r_i = r_(i−1)·2^8 − s_i,
//   so x' = s0·2^-7 + Σ_(i=1..5) s_i·2^(−7−8i) + r5·2^-47: 47 bits, every
//   element within 2^23 of its row's largest is represented exactly, and the
//   truncation is below 2^(e−47) (slicing rounds down);
//
//   the product of slices i of A and j of B is an exact integer (int8 MMA,
//   s32 accumulation); pairs of one level L = i + j (weight 2^(−14−8L)) share
//   one s32 accumulator in TMEM; levels 0..6 (26 pairs) are kept;
//
//   ŷ = 2^(ea+eb−62)·(2^32·((Q0·256 + Q1)·256 + Q2) + ((Q3·256 + Q4)·256 + Q5)·256 + Q6):
//   both parts are exact 64-bit integers below 2^51 (K ≤ 384), converted to
//   f64 exactly (a bit-pattern add and one subtraction), so forming ŷ rounds
//   once.
//
// The bound E per output (all terms rounded up, then doubled, which covers
// the f64 rounding of the bound itself and of ŷ ± E):
//   E1 slicing    2^(ea−47)·‖b‖₁ + 2^(eb−47)·(‖a‖₁ + K·2^(ea−47))
//   E2 levels 7-10 (pairs i, j ∈ [2, 5]): K·255²·Σ_L n_L·2^(−14−8L)·2^(ea+eb)
//   E3 forming ŷ  2^-53·|ŷ|
//   E4 the chain  γ_(K−1)·‖a‖₂·‖b‖₂   (Σ|a_k b_k| ≤ ‖a‖₂‖b‖₂)
// A row with a non-finite entry cannot be sliced: every output it touches
// goes to the fixup. A list that overflows raises an error bit; the caller
// then recomputes the whole forward on the FP64 kernel.
//
// One persistent CTA per SM, 320 threads:
//   warp 0     TMA: per (128-row, 64-column) tile and 128-wide K chunk the
//              six B slices (8 KB each) into a two-deep ring, then the six A
//              slices (16 KB each) into a five-deep ring (3-D tensor maps over
//              [slice][row][k] int8, 128-byte swizzle, zero fill past M);
//   warp 1     MMA issuer: for A slice i, B slices j ≤ 6 − i into level i + j
//              (four K steps of 32 each), s32 accumulators in TMEM;
//   warps 2-9  epilogue: one output row per thread, two warps per TMEM lane
//              quarter (32 columns each), 16 columns at a time. The bound's
//              row terms are formed once per tile, the column terms once per
//              sync (k_oz_slice on the weights), so an output costs three
//              FMAs of bound and two f64 -> f32 conversions. The tile passes
//              through shared memory (float4 group c of row r at
//              c ^ (r & 7)), so the residual or gate input comes in and the
//              results leave with coalesced 16-byte accesses.
#pragma once
#include "common.cuh"
#include "tc_gemm.cuh"

namespace kc {
namespace oz {

using tc::smem_u32;

constexpr int kSlices = 6;
constexpr int kLevels = 7;                       // L = 0..6 kept
constexpr int kBM = 128, kBN = 64, kBK = 128;    // tile rows, tile columns, K bytes per chunk
constexpr int kASlot = kBM * kBK;                // 16 KB: one A slice of one chunk
constexpr int kBSlice = kBN * kBK;               // 8 KB: one B slice of one chunk
constexpr int kBSlot = kSlices * kBSlice;        // 48 KB
constexpr int kAStages = 5, kBStages = 2;
constexpr int kThreads = 320;                    // TMA warp, MMA warp, 8 epilogue warps
constexpr int kStage = kBM * kBN * 4;             // 32 KB: the output tile, f32
constexpr int kColBytes = 3 * kBN * 8;           // the tile's column terms: 2^eb, the bound's term, ‖b‖₂
constexpr int kSmem = kAStages * kASlot + kBStages * kBSlot + kStage + kColBytes + 1024 + 256;
constexpr uint32_t kTmemCols = 512;              // 7 levels x 64 columns used
constexpr int kSpecial = 0x7fffffff;             // a row with a non-finite entry
constexpr int kMaxK = 384;                       // keeps both 64-bit parts of ŷ below 2^51
// Error bits of the product's own word: an expired pipeline wait raises
// tc::kErrTimeout (1), a full list kOzListFull.
enum : int { kOzListFull = 4 };

// ---------------------------------------------------------------------------
// Slicing: one warp per row of X [rows, K] (row stride ldx, 16-byte aligned
// rows, K % 128 == 0). Slice i of row r lands at slices + i·plane + r·K.
// ---------------------------------------------------------------------------
struct SliceArgs {
  const float* X;
  uint64_t rows;
  int K;
  uint64_t ldx;
  uint8_t* slices;
  uint64_t plane;          // rows·K (the slice stride)
  int* e;                  // [rows]
  double* l1;              // [rows] Σ|x|, rounded up
  double* l2;              // [rows] sqrt(Σ x²), rounded up
  unsigned* reset;         // optional: zeroed by the first thread (the next GEMM's list count)
  // weights only (the product's columns): 2^e, and the column's part of the
  // bound 2^-47·‖b‖₁ + c2k·2^e (c2k = K·2^-94 + E2's factor); a column with a
  // non-finite entry gets 0 and +inf, which lists every output it touches
  double* col_s = nullptr;
  double* col_p = nullptr;
  double c2k = 0.0;
};

// 2^x as an f64, exactly, for −1022 ≤ x ≤ 1023.
__device__ __forceinline__ double pow2(int x) { return __longlong_as_double(static_cast<long long>(x + 1023) << 52); }

// floor(x·2^(47−e)) for an f32 x with |x| < 2^e, from its bits (|result| <
// 2^47). Its bytes are the six slices: s0 = result >> 40 (arithmetic: the
// floor), s_i = (result >> (40 − 8i)) & 255, the same digits as slicing
// x·2^-e by repeated floors, since the dropped fraction is below one.
__device__ __forceinline__ long long fixed47(float x, int e) {
  const uint32_t b = __float_as_uint(x);
  const uint32_t ex = (b >> 23) & 0xffu, fr = b & 0x7fffffu;
  if (ex == 0 && fr == 0) return 0;
  const unsigned long long m = ex ? (fr | 0x800000u) : fr;  // |x| = m·2^p
  const int sh = (ex ? int(ex) : 1) - 150 + 47 - e;         // |x|·2^(47−e) = m·2^sh, sh ≤ 23
  unsigned long long mag;
  bool inexact = false;
  if (sh >= 0) {
    mag = m << sh;
  } else if (sh > -64) {
    mag = m >> (-sh);
    inexact = (m & ((1ull << (-sh)) - 1ull)) != 0ull;
  } else {
    mag = 0;
    inexact = true;
  }
  const long long v = static_cast<long long>(mag);
  return (b >> 31) ? -(v + (inexact ? 1 : 0)) : v;  // floor of a negative value
}

// A 64-bit integer below 2^51 in magnitude as an f64, exactly, without the
// conversion pipe: added into the significand of 1.5·2^52, then 1.5·2^52
// subtracted (both steps exact).
__device__ __forceinline__ double i64_to_f64(long long v) {
  return __longlong_as_double(0x4338000000000000LL + v) - 6755399441055744.0;
}

__global__ void __launch_bounds__(256) k_oz_slice(SliceArgs a) {
  if (a.reset && blockIdx.x == 0 && threadIdx.x == 0) *a.reset = 0u;
  const int lane = threadIdx.x & 31;
  const uint64_t r = uint64_t(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (r >= a.rows) return;
  const float* x = a.X + r * a.ldx;
  const int chunks = a.K / 128;  // each lane holds 4 consecutive elements per 128-wide chunk
  float4 v[kMaxK / 128];
  float mx = 0.0f;
  bool bad = false;
  double s1 = 0.0, s2 = 0.0;
#pragma unroll
  for (int c = 0; c < kMaxK / 128; c++) {
    if (c >= chunks) break;
    v[c] = *reinterpret_cast<const float4*>(x + c * 128 + lane * 4);
    const float t[4] = {v[c].x, v[c].y, v[c].z, v[c].w};
#pragma unroll
    for (int q = 0; q < 4; q++) {
      const float m = fabsf(t[q]);
      bad |= !(m <= 3.4028234663852886e38f);  // inf or NaN
      mx = fmaxf(mx, m);
      const double d = double(m);
      s1 += d;
      s2 = fma(d, d, s2);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    bad |= __shfl_xor_sync(0xffffffffu, int(bad), o) != 0;
    s1 += __shfl_xor_sync(0xffffffffu, s1, o);
    s2 += __shfl_xor_sync(0xffffffffu, s2, o);
  }
  int e = 0;
  if (bad) e = kSpecial;
  else if (mx > 0.0f) e = ilogbf(mx) + 1;  // 2^(e-1) <= max < 2^e
  if (lane == 0) {
    a.e[r] = e;
    // the sums' own rounding (at most K·u relative) is covered by the factor
    const double l1 = bad ? 0.0 : s1 * (1.0 + 0x1p-40);
    a.l1[r] = l1;
    a.l2[r] = bad ? 0.0 : sqrt(s2) * (1.0 + 0x1p-40);
    if (a.col_s) {
      a.col_s[r] = bad ? 0.0 : pow2(e);
      a.col_p[r] = bad ? __longlong_as_double(0x7ff0000000000000LL) : fma(a.c2k, pow2(e), l1 * 0x1p-47);
    }
  }
#pragma unroll
  for (int c = 0; c < kMaxK / 128; c++) {
    if (c >= chunks) break;
    const float t[4] = {v[c].x, v[c].y, v[c].z, v[c].w};
    uint32_t w[kSlices] = {0, 0, 0, 0, 0, 0};
    if (!bad && mx > 0.0f) {
#pragma unroll
      for (int q = 0; q < 4; q++) {
        const long long X = fixed47(t[q], e);
        w[0] |= (uint32_t(X >> 40) & 0xffu) << (8 * q);
#pragma unroll
        for (int i = 1; i < kSlices; i++) w[i] |= (uint32_t(X >> (40 - 8 * i)) & 0xffu) << (8 * q);
      }
    }
    uint8_t* dst = a.slices + r * uint64_t(a.K) + c * 128 + lane * 4;
#pragma unroll
    for (int i = 0; i < kSlices; i++) *reinterpret_cast<uint32_t*>(dst + i * a.plane) = w[i];
  }
}

// ---------------------------------------------------------------------------
// The product.
// ---------------------------------------------------------------------------
struct GemmArgs {
  int M, N, K;
  const int* ea;                // A rows: exponent, ‖a‖₁, ‖a‖₂
  const double *l1a, *l2a;
  const double *sb, *pb, *l2b;  // B rows (the output columns): 2^eb, the bound's column term, ‖b‖₂
  float* C;
  int ldc;
  const float* gate;            // kEpiGate: [M, ldc]
  unsigned long long* list;     // flagged outputs: row << 32 | column
  unsigned* count;
  unsigned cap;
  int* err;                     // tc::kErrTimeout / kOzListFull
  double gamma;                 // γ_(K−1)
  int inject_expiry;            // test hook: the producer reports an expired wait before it issues any copy
};

// Instruction descriptor: D s32, A / B int8 (signed for slice 0), K-major,
// M = 128, N = 64 or 128.
__host__ __device__ constexpr uint32_t idesc_i8(bool a_signed, bool b_signed, int n) {
  return (2u << 4) | (uint32_t(a_signed) << 7) | (uint32_t(b_signed) << 10) | (uint32_t(n >> 3) << 17) |
         (uint32_t(kBM >> 4) << 24);
}

// The order the A slices are loaded and multiplied in: slice 1 first, so that
// its products write levels 1-6 fresh, then slice 0 (level 0 fresh, the rest
// accumulating), then 2..5.
__device__ __forceinline__ int slice_at(int idx) { return idx == 0 ? 1 : idx == 1 ? 0 : idx; }

__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
  const uint32_t z = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(z), "r"(z), "r"(z), "r"(z)
      : "memory");
}

// 3-D TMA load of one slice's [rows x 128 bytes] box at (k, row, slice).
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

// 32 lanes x 16 columns of 32-bit words from TMEM, without the wait.
__device__ __forceinline__ void tmem_ld16_async(uint32_t taddr, int* v) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// One output's decision: the stored f32 (true) or a listing (false). Row
// terms: sr = 2^(ea−62), ar = 2^ea, br = 2^-47·‖a‖₁, cr = γ·‖a‖₂ (a row with a
// non-finite entry: sr = 0, ar = +inf, so it is always listed). With the
// column terms the bound is
//   E = 2·(ar·pb + br·sb + cr·‖b‖₂ + 2^-53·|ŷ|) = 2·(E1 + E2 + E4 + E3).
__device__ __forceinline__ bool oz_decide(const int* q, double sr, double ar, double br, double cr, double sb,
                                          double pb, double l2b, float* out) {
  // (no early exit: the caller keeps its loop free of branches)
  const long long hi = (static_cast<long long>(q[0]) * 256 + q[1]) * 256 + q[2];
  const long long lo = ((static_cast<long long>(q[3]) * 256 + q[4]) * 256 + q[5]) * 256 + q[6];
  const double y = fma(i64_to_f64(hi), 0x1p32, i64_to_f64(lo)) * (sr * sb);
  double t = fma(cr, l2b, fabs(y) * 0x1p-53);
  t = fma(br, sb, t);
  t = fma(ar, pb, t);
  const double err = 2.0 * t + 0x1p-1060;  // (the last term: a scale that went subnormal)
  const float lo_f = __double2float_rn(y - err), hi_f = __double2float_rn(y + err);
  *out = lo_f;
  return __float_as_uint(lo_f) == __float_as_uint(hi_f);
}

template <int EPI>
__global__ void __launch_bounds__(kThreads, 1) k_oz_gemm(const __grid_constant__ CUtensorMap amap,
                                                         const __grid_constant__ CUtensorMap bmap, GemmArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* aring = smem;
  unsigned char* bring = smem + kAStages * kASlot;
  float4* stage = reinterpret_cast<float4*>(bring + kBStages * kBSlot);  // [128 rows][16 float4]
  double* colsm = reinterpret_cast<double*>(bring + kBStages * kBSlot + kStage);  // [3][64]
  uint64_t* bars = reinterpret_cast<uint64_t*>(bring + kBStages * kBSlot + kStage + kColBytes);
  uint64_t* afull = bars;
  uint64_t* aempty = afull + kAStages;
  uint64_t* bfull = aempty + kAStages;
  uint64_t* bempty = bfull + kBStages;
  uint64_t* tfull = bempty + kBStages;
  uint64_t* tempty = tfull + 1;
  uint64_t* drain = tempty + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m_tiles = (a.M + kBM - 1) / kBM, n_tiles = a.N / kBN;
  const int tiles = m_tiles * n_tiles;
  const int chunks = a.K / kBK;
  int* perr = a.err;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kAStages; s++) {
      tc::mbar_init(&afull[s], 1);
      tc::mbar_init(&aempty[s], 1);
    }
    for (int s = 0; s < kBStages; s++) {
      tc::mbar_init(&bfull[s], 1);
      tc::mbar_init(&bempty[s], 1);
    }
    tc::mbar_init(tfull, 1);
    tc::mbar_init(tempty, 256);
    tc::mbar_init(drain, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) tc::tmem_alloc(tmem_slot, kTmemCols);
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA issuer ----------------
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&amap)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&bmap)) : "memory");
      uint32_t ai = 0, bi = 0;
      bool ok = true;
      if (a.inject_expiry) {  // as if the first wait had expired: nothing is issued
        atomicOr(perr, tc::kErrTimeout);
        ok = false;
      }
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        const int m = t / n_tiles, n = t % n_tiles;
        for (int c = 0; c < chunks && ok; c++) {
          {
            const int s = bi % kBStages;
            const uint32_t ph = (bi / kBStages) & 1;
            if (!tc::mbar_wait(&bempty[s], ph ^ 1, perr)) { ok = false; break; }
            tc::mbar_arrive_expect_tx(&bfull[s], kBSlot);
            for (int j = 0; j < kSlices; j++)
              tma_load_3d(bring + s * kBSlot + j * kBSlice, &bmap, c * kBK, n * kBN, j, &bfull[s]);
            bi++;
          }
          for (int idx = 0; idx < kSlices; idx++, ai++) {
            const int s = ai % kAStages;
            const uint32_t ph = (ai / kAStages) & 1;
            if (!tc::mbar_wait(&aempty[s], ph ^ 1, perr)) { ok = false; break; }
            tc::mbar_arrive_expect_tx(&afull[s], kASlot);
            tma_load_3d(aring + s * kASlot, &amap, c * kBK, m * kBM, slice_at(idx), &afull[s]);
          }
        }
      }
      // every copy issued lands before the CTA may exit
      for (uint32_t j = ai > uint32_t(kAStages) ? ai - kAStages : 0u; j < ai; j++)
        tc::mbar_wait_drain(&afull[j % kAStages], (j / kAStages) & 1);
      for (uint32_t j = bi > uint32_t(kBStages) ? bi - kBStages : 0u; j < bi; j++)
        tc::mbar_wait_drain(&bfull[j % kBStages], (j / kBStages) & 1);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      uint32_t ai = 0, bi = 0, tl = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, tl++) {
        if (!tc::mbar_wait(tempty, (tl & 1) ^ 1, perr)) { ok = false; break; }
        tc::tc_fence_after();
        uint32_t started = 0;  // levels written in this tile
        for (int c = 0; c < chunks && ok; c++) {
          const int bs = bi % kBStages;
          if (!tc::mbar_wait(&bfull[bs], (bi / kBStages) & 1, perr)) { ok = false; break; }
          tc::tc_fence_after();
          const uint32_t bb = smem_u32(bring + bs * kBSlot);
          for (int idx = 0; idx < kSlices; idx++, ai++) {
            const int i = slice_at(idx);
            const int as = ai % kAStages;
            if (!tc::mbar_wait(&afull[as], (ai / kAStages) & 1, perr)) { ok = false; break; }
            tc::tc_fence_after();
            const uint32_t ab = smem_u32(aring + as * kASlot);
            // B slice 0 (signed) alone; the unsigned slices j, j+1 two at a
            // time as one N = 128 product: B slices j and j+1 are adjacent in
            // shared memory, levels i+j and i+j+1 adjacent in TMEM, and both
            // levels are fresh or both accumulating (the order above)
            const int jmax = kLevels - 1 - i < kSlices - 1 ? kLevels - 1 - i : kSlices - 1;
            for (int j = 0; j <= jmax;) {
              const int wide = (j > 0 && j + 1 <= jmax) ? 2 : 1;
              const int L = i + j;
              const uint32_t id = idesc_i8(i == 0, j == 0, kBN * wide);
              const uint32_t d = tmem_base + uint32_t(L * kBN);
              const uint32_t acc = (started >> L) & 1u;
#pragma unroll
              for (int kk = 0; kk < kBK / 32; kk++)
                mma_i8(d, tc::smem_desc(ab + kk * 32), tc::smem_desc(bb + j * kBSlice + kk * 32), id,
                       acc | uint32_t(kk > 0));
              started |= (wide == 2 ? 3u : 1u) << L;
              j += wide;
            }
            tc::mma_commit(&aempty[as]);
          }
          if (!ok) break;
          tc::mma_commit(&bempty[bs]);
          bi++;
        }
        if (!ok) break;
        tc::mma_commit(tfull);
      }
      tc::mma_commit(drain);
      tc::mbar_wait_drain(drain, 0);
    }
    __syncwarp();
  } else {
    // ---------------- epilogue: one row per thread ----------------
    const int g = warp & 3;             // this warp's TMEM lane quarter
    const int half = (warp - 2) >> 2;   // its 32 columns of the tile
    const int et = threadIdx.x - 64;    // 0..255 among the epilogue threads
    const int rl = g * 32 + lane;       // this thread's row in the tile
    uint32_t tl = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, tl++) {
      const int m = t / n_tiles, n = t % n_tiles;
      int okw = 0;
      if (lane == 0) okw = tc::mbar_wait(tfull, tl & 1, perr) ? 1 : 0;
      okw = __shfl_sync(0xffffffffu, okw, 0);
      // the eight warps agree before any of them reaches a named barrier
      int all;
      asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %1, 0;\n\t"
                   "bar.red.and.pred p, 1, 256, p;\n\tselp.u32 %0, 1, 0, p;\n\t}"
                   : "=r"(all) : "r"(okw) : "memory");
      if (!all) break;
      tc::tc_fence_after();
      const int row = m * kBM + rl;
      const bool live = row < a.M;
      double sr = 0.0, ar = 0.0, br = 0.0, cr = 0.0;
      if (live) {
        const int ea = a.ea[row];
        if (ea == kSpecial) {
          ar = __longlong_as_double(0x7ff0000000000000LL);
        } else {
          sr = pow2(ea - 62);
          ar = pow2(ea);
          br = a.l1a[row] * 0x1p-47;
          cr = a.gamma * a.l2a[row];
        }
      }
      if (et < kBN) {  // the tile's column terms, read by every row
        colsm[et] = a.sb[n * kBN + et];
        colsm[kBN + et] = a.pb[n * kBN + et];
        colsm[2 * kBN + et] = a.l2b[n * kBN + et];
      }
      if (EPI == kEpiResid || EPI == kEpiGate) {  // the residual / gate tile, coalesced
        const float* src = EPI == kEpiGate ? a.gate : a.C;
        for (int i = et; i < kBM * 16; i += 256) {
          const int r = i >> 4, c4 = i & 15;
          const int64_t gr = int64_t(m) * kBM + r;
          float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
          if (gr < a.M) v = *reinterpret_cast<const float4*>(src + gr * a.ldc + n * kBN + c4 * 4);
          stage[r * 16 + (c4 ^ (r & 7))] = v;
        }
      }
      asm volatile("bar.sync 1, 256;" ::: "memory");
#pragma unroll 1
      for (int cc = 0; cc < 2; cc++) {
        int q[kLevels][16];
        const int c0 = half * 32 + cc * 16;  // the chunk's first column in the tile
        const uint32_t base = tmem_base + (uint32_t(g * 32) << 16) + uint32_t(c0);
#pragma unroll
        for (int L = 0; L < kLevels; L++) tmem_ld16_async(base + uint32_t(L * kBN), q[L]);
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        if (cc == 1) {  // this warp's accumulators are read: once all eight are, the next tile may start
          tc::tc_fence_before();
          tc::mbar_arrive(tempty);
        }
        uint32_t listed = 0;  // bit e: output e of this chunk goes to the fixup
#pragma unroll
        for (int gq = 0; gq < 4 && live; gq++) {
          float4* sp = stage + rl * 16 + (((c0 >> 2) + gq) ^ (rl & 7));
          const float4 cur = *sp;  // the residual or gate input (a listed output keeps it)
          float o[4] = {cur.x, cur.y, cur.z, cur.w};
#pragma unroll
          for (int u = 0; u < 4; u++) {
            const int e = gq * 4 + u;
            const int cl = c0 + e;  // column in the tile
            const int qe[kLevels] = {q[0][e], q[1][e], q[2][e], q[3][e], q[4][e], q[5][e], q[6][e]};
            float v;
            const bool ok = oz_decide(qe, sr, ar, br, cr, colsm[cl], colsm[kBN + cl], colsm[2 * kBN + cl], &v);
            float r;
            if (EPI == kEpiStore) r = v;
            else if (EPI == kEpiRelu) r = js_relu(v);
            else if (EPI == kEpiGate) r = o[u] > 0.0f ? v : 0.0f;
            // f32(double(c) + double(v)), the oracle's addInPlace: rounding the
            // exact sum to f64 and then to f32 equals rounding it to f32 once
            // (double rounding is innocuous for a sum when 53 >= 2·24 + 2)
            else r = __fadd_rn(o[u], v);
            o[u] = ok ? r : o[u];
            listed |= ok ? 0u : 1u << e;
          }
          *sp = make_float4(o[0], o[1], o[2], o[3]);
        }
        if (__any_sync(0xffffffffu, listed != 0)) {  // every lane votes (a row past M lists nothing)
          while (listed) {
            const int e = __ffs(listed) - 1;
            listed &= listed - 1;
            const int col = n * kBN + c0 + e;
            const unsigned slot = atomicAdd(a.count, 1u);
            if (slot < a.cap) a.list[slot] = (static_cast<unsigned long long>(row) << 32) | unsigned(col);
            else atomicOr(a.err, kOzListFull);
          }
        }
      }
      asm volatile("bar.sync 1, 256;" ::: "memory");
      for (int i = et; i < kBM * 16; i += 256) {  // the tile leaves coalesced
        const int r = i >> 4, c4 = i & 15;
        const int64_t gr = int64_t(m) * kBM + r;
        if (gr < a.M) *reinterpret_cast<float4*>(a.C + gr * a.ldc + n * kBN + c4 * 4) = stage[r * 16 + (c4 ^ (r & 7))];
      }
      asm volatile("bar.sync 1, 256;" ::: "memory");  // the stage is free for the next tile
    }
  }

  tc::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem_base, kTmemCols);
  }
}

// The listed outputs by the sequential f64 chain, as k_dgemm_exact computes
// them, with the same epilogue. Grid-stride over the list.
struct FixupArgs {
  const float* A;
  uint64_t lda;
  const float* B;
  uint64_t ldb;
  int K;
  float* C;
  int ldc;
  const float* gate;
  const unsigned long long* list;
  const unsigned* count;
  unsigned cap;
  unsigned long long* listed;   // running total of listed outputs (profile counter)
};

// The sequential f64 chain of one listed output in k order, as k_dgemm_exact
// forms it, and its store through the product's epilogue.
template <int EPI>
__device__ __forceinline__ void oz_fix_store(const FixupArgs& a, uint64_t row, int col, double acc) {
  const float v = f32(acc);
  float* cp = a.C + row * uint64_t(a.ldc) + col;
  if (EPI == kEpiStore) *cp = v;
  else if (EPI == kEpiRelu) *cp = js_relu(v);
  else if (EPI == kEpiGate) *cp = a.gate[row * uint64_t(a.ldc) + col] > 0.0f ? v : 0.0f;
  else *cp = f32(double(*cp) + double(v));
}

// Many listed outputs (more than 8 per warp of the grid): a thread per
// output, its row loads inside the chain, latency hidden by the other
// threads. Few (the frames a certified batch recomputes): a warp per output,
// the lanes bringing its A row and B row into shared memory with coalesced
// loads (one round trip), lane 0 running the chain over them. Either way the
// same chain, so the same bits.
template <int EPI>
__global__ void __launch_bounds__(256) k_oz_fixup(FixupArgs a) {
  __shared__ float4 rows[8][2][kMaxK / 4];  // per warp: the A row, the B row
  const unsigned n = min(*a.count, a.cap);
  if (blockIdx.x == 0 && threadIdx.x == 0) atomicAdd(a.listed, static_cast<unsigned long long>(n));
  if (n > gridDim.x * 64u) {
    for (unsigned i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
      const unsigned long long ent = a.list[i];
      const uint64_t row = ent >> 32;
      const int col = int(ent & 0xffffffffu);
      const float* ar = a.A + row * a.lda;
      const float* br = a.B + uint64_t(col) * a.ldb;
      double acc = 0.0;
      for (int k = 0; k < a.K; k += 4) {
        const float4 x = *reinterpret_cast<const float4*>(ar + k);
        const float4 w = *reinterpret_cast<const float4*>(br + k);
        acc = fma(double(x.x), double(w.x), acc);
        acc = fma(double(x.y), double(w.y), acc);
        acc = fma(double(x.z), double(w.z), acc);
        acc = fma(double(x.w), double(w.w), acc);
      }
      oz_fix_store<EPI>(a, row, col, acc);
    }
    return;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int k4 = a.K / 4;
  for (unsigned i = blockIdx.x * 8 + warp; i < n; i += gridDim.x * 8) {
    const unsigned long long ent = a.list[i];
    const uint64_t row = ent >> 32;
    const int col = int(ent & 0xffffffffu);
    const float4* ar = reinterpret_cast<const float4*>(a.A + row * a.lda);
    const float4* br = reinterpret_cast<const float4*>(a.B + uint64_t(col) * a.ldb);
    for (int k = lane; k < k4; k += 32) {
      rows[warp][0][k] = ar[k];
      rows[warp][1][k] = br[k];
    }
    __syncwarp();
    if (lane == 0) {
      double acc = 0.0;
      for (int k = 0; k < k4; k++) {
        const float4 x = rows[warp][0][k], w = rows[warp][1][k];
        acc = fma(double(x.x), double(w.x), acc);
        acc = fma(double(x.y), double(w.y), acc);
        acc = fma(double(x.z), double(w.z), acc);
        acc = fma(double(x.w), double(w.w), acc);
      }
      oz_fix_store<EPI>(a, row, col, acc);
    }
    __syncwarp();  // the rows are read before the next output's land
  }
}

// E2's factor: K·255²·Σ_(L=7..10) n_L·2^(−14−8L), n_L = 11 − L pairs of slices
// i, j ∈ [2, 5] with i + j = L. The weights' column term adds E1's K·2^-94.
inline double dropped_levels_bound(int K) {
  double s = 0.0;
  for (int L = 7; L <= 10; L++) s += double(11 - L) * std::ldexp(1.0, -14 - 8 * L);
  return double(K) * 65025.0 * s;
}

inline double chain_gamma(int K) {
  const double nu = double(K - 1) * std::ldexp(1.0, -53);
  return nu / (1.0 - nu);
}

// The tensor map of slices [6][rows][K] int8: boxes of [box_rows x 128 bytes]
// of one slice, 128-byte swizzle, zero fill past the last row.
inline bool make_slice_map(CUtensorMap* map, const uint8_t* base, uint64_t rows, uint64_t K, uint32_t box_rows) {
  tc::EncodeTiledFn fn = tc::encode_tiled_fn();
  if (!fn || (reinterpret_cast<uintptr_t>(base) & 15) || K % 128 || rows == 0) return false;
  const cuuint64_t dims[3] = {K, rows, uint64_t(kSlices)};
  const cuuint64_t strides[2] = {K, rows * K};
  const cuuint32_t box[3] = {uint32_t(kBK), box_rows, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<uint8_t*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace oz
}  // namespace kc
