// tc_gemm.cuh — y = x·Wᵀ on the 5th-generation tensor cores (tcgen05).
//
// fp32-class precision from fp16 tensor cores by splitting both operands
// (Ootomo & Yokota, "Recovering single precision accuracy from Tensor Cores
// while surpassing the FP32 theoretical peak performance", IJHPCA 2022):
// x·2^sa = xh + xl and W·2^sw = Wh + Wl with xh = fp16(x·2^sa),
// xl = fp16(x·2^sa − xh), and y·2^(sa+sw) ≈ xh·Whᵀ + xh·Wlᵀ + xl·Whᵀ, all three
// products accumulated in one fp32 TMEM accumulator (the dropped xl·Wlᵀ term
// is ~2^-22 relative). Powers of two keep the scaling exact.
//
// One persistent CTA per SM, warp-specialised:
//   warp 0     TMA issuer: a 2-D tensor-map load of the [128 x 64] f32 chunk
//              of A and bulk copies of the matching pre-swizzled weight tiles.
//   warps 1-4  split the staged f32 chunk into swizzled fp16 hi/lo tiles.
//   warp 5     MMA issuer: 12 tcgen05.mma (4 K-steps x 3 products) per chunk
//              into a 128x128 fp32 accumulator in TMEM; tcgen05.commit frees
//              the stage; two accumulators double-buffer the epilogue.
//   warps 6-9  epilogue: tcgen05.ld the accumulator rows, unscale, apply
//              store / ReLU / residual in 128-byte swizzled shared tiles,
//              TMA-store them (the residual input arrives by TMA load).
// Every wait is bounded (about two seconds); on expiry the kernel raises the
// error word and drains, so a fault in the pipeline can never hang the GPU.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>

#include "common.cuh"

namespace kc {
namespace tc {

constexpr int kBM = 128;         // rows per tile (TMEM lanes)
constexpr int kBN = 128;         // columns per tile (TMEM columns per accumulator)
constexpr int kBK = 64;          // K per chunk: one 128-byte swizzle row of fp16
constexpr int kTileBytes = kBM * kBK * 2;           // 16 KB: one fp16 [128 x 64] tile
constexpr uint32_t kTmemCols = 2 * kBN;              // two accumulators
constexpr long long kWaitCycles = 4000000000ll;      // ~2 s per wait at the B200's clocks

// Error word bits.
enum : int { kErrTimeout = 1, kErrOverflow = 2 };

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait on a phase parity. Returns false (and raises the error word)
// when the budget expires or another thread has already raised it. The loop
// stays tight: the error word (a global load) and the SM clock are looked at
// once every 64 failed tries, so a completed phase is seen at once.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  for (uint32_t i = 1;; i++) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63u) == 0) {
      if (*reinterpret_cast<volatile int*>(err) & kErrTimeout) return false;
      if (clock64() - t0 > kWaitCycles) {
        atomicOr(err, kErrTimeout);
        return false;
      }
    }
  }
}

// Wait for copies or MMAs already issued before the CTA leaves: bounded by
// the clock alone. It does not give up when the error word is raised, since
// a copy still landing in shared memory, or an MMA still using TMEM, must
// finish before the CTA exits or frees TMEM. An issued copy or MMA always
// completes, so the bound is only a backstop.
__device__ __forceinline__ void mbar_wait_drain(uint64_t* bar, uint32_t parity) {
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity))
    if (clock64() - t0 > kWaitCycles) return;
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// 1-D bulk copy global -> shared (the TMA engine), completing on an mbarrier.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row atoms of
// 1024 bytes (stride byte offset 1024), descriptor version 1.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= uint64_t((saddr >> 4) & 0x3FFFu);          // start address
  d |= uint64_t(1) << 16;                         // leading byte offset (unused with 128B swizzle)
  d |= uint64_t(1024 >> 4) << 32;                 // stride byte offset
  d |= uint64_t(1) << 46;                         // version
  d |= uint64_t(2) << 61;                         // SWIZZLE_128B
  return d;
}

// Instruction descriptor: D f32, A/B f16, both K-major, M = 128, N = 128.
constexpr uint32_t kIdesc = (1u << 4) | (0u << 7) | (0u << 10) | (uint32_t(kBN >> 3) << 17) | (uint32_t(kBM >> 4) << 24);

__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  const uint32_t z = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(accumulate), "r"(z), "r"(z), "r"(z), "r"(z)
      : "memory");
}

// The same product with A read from TMEM (M = 128 rows in lanes 0-127, K
// consecutive fp16 packed two per 32-bit column, 8 columns per K step of 16).
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t accumulate) {
  const uint32_t z = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(kIdesc), "r"(accumulate), "r"(z), "r"(z), "r"(z), "r"(z)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// tcgen05.wait::ld that names the 32 destination registers of a load, so no
// use of them can be scheduled before the wait.
__device__ __forceinline__ void tmem_wait_regs(uint32_t* r) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                 "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                 "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}

// 32 lanes x 32 columns of f32 from TMEM (this warp's lane quarter).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  tmem_wait_regs(r);
#pragma unroll
  for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
}

// The same load without the wait: tmem_ld_wait() before reading v.
__device__ __forceinline__ void tmem_ld32_async(uint32_t taddr, float* v) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait(float* v) { tmem_wait_regs(reinterpret_cast<uint32_t*>(v)); }

// 32 lanes x 32 columns of 32-bit words into TMEM (this warp's lane quarter);
// tmem_st_wait() before anything reads them.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
      ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
        "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
        "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Veltkamp split (Dekker 1971): hi keeps the leading 11 significant bits of x
// (exactly representable in fp16 for |x| >= 2^-14), lo = x - hi is exact in
// f32 and is rounded once when converted to fp16.
__device__ __forceinline__ void split_f32(float x, float& hi, float& lo) {
  const float t = __fmul_rn(x, 8193.0f);  // 2^13 + 1
  hi = __fsub_rn(t, __fsub_rn(t, x));
  lo = __fsub_rn(x, hi);
}

__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

// Byte offset of element (row, k) of a [rows x 64] fp16 tile in the
// 128-byte-swizzled K-major layout the descriptor above describes.
__device__ __forceinline__ uint32_t swz_offset(uint32_t row, uint32_t k) {
  const uint32_t byte = k * 2;
  return (row >> 3) * 1024 + (row & 7) * 128 + ((((byte >> 4) ^ (row & 7)) & 7) << 4) + (byte & 15);
}

// Epilogues: store, ReLU, residual add (C += acc, C loaded by TMA), and the
// ReLU backward gate (C = gate > 0 ? acc : 0, the gate [M, N] loaded by TMA).
enum { kEpiStore = 0, kEpiRelu = 1, kEpiResid = 2, kEpiGate = 3 };

constexpr int kMaxPlanes = 8;

struct GemmArgs {
  int M, K;
  int n_sub;             // N / 128
  const uint8_t* B;      // weight images: [n_sub][K/64][hi 16 KB | lo 16 KB]
  float* C;              // [M, N] f32, row stride ldc
  int ldc;
  float a_scale;         // 2^sa
  float unscale;         // 2^-(sa+sw)
  int* err;              // error word
  int inject_expiry;     // test hook: the producer reports an expired wait before it issues any copy
  // kEpiStore over the matrices of one input (planes > 0, the matrices'
  // count, one or more): n-tile p is matrix p, scaled by unscale_n[p] and
  // stored to plane p of a [planes, M, 128] output through a 3-D map, as
  // separate products would store them; 0: an ordinary product
  int planes;
  float unscale_n[kMaxPlanes];
};

// 2-D TMA load of a [128 rows x 64 f32] box of A (no swizzle) at (x = k, y = row).
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

constexpr int kStagesT = 3;
// A region (32 KB: the TMA lands f32 there, the split rewrites it in place as
// fp16 hi | lo) then B hi | B lo (32 KB)
constexpr int kStageBytesT = 4 * kTileBytes;
constexpr int kEpiBuf = 32 * 32 * 4;           // one 32x32 f32 block, 128-byte swizzled rows
constexpr int kEpiBytes = 4 * 2 * kEpiBuf;      // two per epilogue warp
constexpr int kSmemBytesT = kStagesT * kStageBytesT + kEpiBytes + 1024 + 256;
constexpr int kThreadsT = 320;                // TMA warp, 4 split warps, MMA warp, 4 epilogue warps

// Warp roles: 0 TMA issuer, 1-4 split A f32 -> fp16 hi/lo, 5 MMA issuer, 6-9 epilogue.
template <int EPI>
__global__ void __launch_bounds__(kThreadsT, 1) k_tc_gemm(const __grid_constant__ CUtensorMap amap,
                                                           const __grid_constant__ CUtensorMap cmap,
                                                           const __grid_constant__ CUtensorMap gmap, GemmArgs a) {
  constexpr bool kLoadTile = EPI == kEpiResid || EPI == kEpiGate;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* epi_buf = reinterpret_cast<float*>(smem + kStagesT * kStageBytesT);
  uint64_t* raw = reinterpret_cast<uint64_t*>(smem + kStagesT * kStageBytesT + kEpiBytes);
  uint64_t* full = raw + kStagesT;
  uint64_t* empty = full + kStagesT;
  uint64_t* tfull = empty + kStagesT;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* cload = drain + 1;  // [4 warps][2 buffers]: residual tiles landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(cload + 8);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m_tiles = (a.M + kBM - 1) / kBM;
  const int tiles = m_tiles * a.n_sub;
  const int kchunks = a.K / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStagesT; s++) {
      mbar_init(&raw[s], 1);
      mbar_init(&full[s], 128);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 128);
    }
    mbar_init(drain, 1);
    for (int i = 0; i < 8; i++) mbar_init(&cload[i], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 5) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA issuer ----------------
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&amap)) : "memory");
      uint32_t it = 0;
      bool ok = true;
      if (a.inject_expiry) {  // as if the first wait had expired: nothing is issued
        atomicOr(a.err, kErrTimeout);
        ok = false;
      }
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        const int m = t / a.n_sub, n = t % a.n_sub;
        for (int kc = 0; kc < kchunks; kc++, it++) {
          const int s = it % kStagesT;
          const uint32_t ph = (it / kStagesT) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, a.err)) { ok = false; break; }
          unsigned char* st = smem + s * kStageBytesT;
          mbar_arrive_expect_tx(&raw[s], 4 * kTileBytes);
          tma_load_2d(st, &amap, kc * kBK, m * kBM, &raw[s]);
          const uint8_t* src = a.B + (size_t(n) * kchunks + kc) * (2 * kTileBytes);
          bulk_g2s(st + 2 * kTileBytes, src, kTileBytes, &raw[s]);
          bulk_g2s(st + 3 * kTileBytes, src + kTileBytes, kTileBytes, &raw[s]);
        }
      }
      // every copy issued must have landed before the CTA may exit (on the
      // normal path the split warps already waited for them: these pass at once)
      for (uint32_t j = it > uint32_t(kStagesT) ? it - kStagesT : 0u; j < it; j++)
        mbar_wait_drain(&raw[j % kStagesT], (j / kStagesT) & 1);
    }
    __syncwarp();
  } else if (warp <= 4) {
    // ---------------- split: f32 staging -> swizzled fp16 hi / lo ----------------
    const int tid = threadIdx.x - 32;
    uint32_t it = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
      bool ok = true;
      for (int kc = 0; kc < kchunks; kc++, it++) {
        const int s = it % kStagesT;
        const uint32_t ph = (it / kStagesT) & 1;
        // every split thread arrives at the named barrier once per chunk, so a
        // wait that expired for some threads stops all of them together
        const int mine = mbar_wait(&raw[s], ph, a.err) ? 1 : 0;
        int all;
        asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %1, 0;\n\t"
                     "bar.red.and.pred p, 1, 128, p;\n\tselp.u32 %0, 1, 0, p;\n\t}"
                     : "=r"(all) : "r"(mine) : "memory");
        if (!all) { ok = false; break; }
        unsigned char* st = smem + s * kStageBytesT;
        // the f32 box is read whole into registers, then overwritten in place
        float4 v[16];
        const float4* stage = reinterpret_cast<const float4*>(st);
#pragma unroll
        for (int i = 0; i < 16; i++) v[i] = stage[i * 128 + tid];  // float4 index in the [128 x 64] box
        asm volatile("bar.sync 1, 128;" ::: "memory");          // the 4 split warps only
        bool bad = false;
#pragma unroll
        for (int i = 0; i < 16; i++) {
          const int L = i * 128 + tid;
          const int r = L >> 4, c4 = L & 15;
          float xs[4] = {v[i].x * a.a_scale, v[i].y * a.a_scale, v[i].z * a.a_scale, v[i].w * a.a_scale};
          float hs[4], ls[4];
#pragma unroll
          for (int e = 0; e < 4; e++) {
            bad |= !(fabsf(xs[e]) < 32768.0f);  // also catches NaN
            split_f32(xs[e], hs[e], ls[e]);
          }
          const __half2 h01 = __floats2half2_rn(hs[0], hs[1]), h23 = __floats2half2_rn(hs[2], hs[3]);
          const __half2 l01 = __floats2half2_rn(ls[0], ls[1]), l23 = __floats2half2_rn(ls[2], ls[3]);
          const uint32_t off = swz_offset(r, c4 * 4);
          *reinterpret_cast<uint2*>(st + off) = make_uint2(h2u(h01), h2u(h23));
          *reinterpret_cast<uint2*>(st + kTileBytes + off) = make_uint2(h2u(l01), h2u(l23));
        }
        if (bad) atomicOr(a.err, kErrOverflow);
        fence_proxy_async_smem();
        mbar_arrive(&full[s]);
      }
      if (!ok) break;
    }
  } else if (warp == 5) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      uint32_t it = 0, tl = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, tl++) {
        const uint32_t acc = tl & 1, aph = (tl >> 1) & 1;
        if (!mbar_wait(&tempty[acc], aph ^ 1, a.err)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d = tmem_base + acc * kBN;
        for (int kc = 0; kc < kchunks; kc++, it++) {
          const int s = it % kStagesT;
          const uint32_t ph = (it / kStagesT) & 1;
          if (!mbar_wait(&full[s], ph, a.err)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sb = smem_u32(smem + s * kStageBytesT);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; kk++) {
            const uint64_t ah = smem_desc(sb + kk * 32);
            const uint64_t al = smem_desc(sb + kTileBytes + kk * 32);
            const uint64_t bh = smem_desc(sb + 2 * kTileBytes + kk * 32);
            const uint64_t bl = smem_desc(sb + 3 * kTileBytes + kk * 32);
            mma_f16(d, ah, bh, (kc > 0 || kk > 0) ? 1u : 0u);
            mma_f16(d, ah, bl, 1u);
            mma_f16(d, al, bh, 1u);
          }
          mma_commit(&empty[s]);
        }
        if (!ok) break;
        mma_commit(&tfull[acc]);
      }
      // every MMA this thread issued completes before TMEM is released
      mma_commit(drain);
      mbar_wait_drain(drain, 0);
    }
    __syncwarp();
  } else {
    // ---------------- epilogue ----------------
    // Each 32x32 accumulator block is written as 128-byte swizzled rows into
    // one of this warp's two shared buffers and leaves with one TMA store;
    // the residual block arrives the same way, by a TMA load.
    const int g = warp & 3;  // TMEM lane quarter this warp may read
    const int ew = warp - 6;
    unsigned char* bufs = reinterpret_cast<unsigned char*>(epi_buf) + ew * 2 * kEpiBuf;
    uint32_t cphase = 0;      // parity bits of this warp's two residual barriers
    uint32_t tl = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, tl++) {
      const int m = t / a.n_sub, n = t % a.n_sub;
      const uint32_t acc = tl & 1, aph = (tl >> 1) & 1;
      // one lane waits, the warp follows: tcgen05.ld below is warp-collective
      int okw = 0;
      if (lane == 0) okw = mbar_wait(&tfull[acc], aph, a.err) ? 1 : 0;
      okw = __shfl_sync(0xffffffffu, okw, 0);
      if (!okw) { ok = false; break; }
      tc_fence_after();
      const int row0 = m * kBM + g * 32;
      float us = a.unscale;
      if (a.planes > 0)
#pragma unroll
        for (int p = 0; p < kMaxPlanes; p++) us = p == n ? a.unscale_n[p] : us;
#pragma unroll 1
      for (int cc = 0; cc < kBN / 32; cc++) {
        const int b = cc & 1;
        unsigned char* buf = bufs + b * kEpiBuf;
        const int x = n * kBN + cc * 32;
        if (lane == 0) {
          // the TMA store that last read this buffer must be done with it
          asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
          if (kLoadTile) {
            const CUtensorMap* lmap = EPI == kEpiGate ? &gmap : &cmap;
            mbar_arrive_expect_tx(&cload[ew * 2 + b], kEpiBuf);
            asm volatile(
                "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
                ::"r"(smem_u32(buf)), "l"(reinterpret_cast<uint64_t>(lmap)), "r"(x), "r"(row0),
                "r"(smem_u32(&cload[ew * 2 + b]))
                : "memory");
          }
        }
        float v[32];
        tmem_ld32(tmem_base + (uint32_t(g * 32) << 16) + acc * kBN + cc * 32, v);
        if (kLoadTile) {  // every lane observes the landing of the tile it reads
          const bool mine = mbar_wait(&cload[ew * 2 + b], (cphase >> b) & 1, a.err);
          if (!__all_sync(0xffffffffu, mine)) {
            // the residual load issued above lands before the CTA may exit
            if (lane == 0) mbar_wait_drain(&cload[ew * 2 + b], (cphase >> b) & 1);
            ok = false;
            break;
          }
          cphase ^= 1u << b;
        }
        // row = lane; 16-byte chunk j of the row sits at chunk j ^ (row & 7)
        unsigned char* rowp = buf + lane * 128;
#pragma unroll
        for (int j = 0; j < 8; j++) {
          float4 o = make_float4(v[4 * j] * us, v[4 * j + 1] * us, v[4 * j + 2] * us, v[4 * j + 3] * us);
          float4* cp = reinterpret_cast<float4*>(rowp + ((j ^ (lane & 7)) << 4));
          if (EPI == kEpiRelu) {
            o.x = fmaxf(o.x, 0.f); o.y = fmaxf(o.y, 0.f); o.z = fmaxf(o.z, 0.f); o.w = fmaxf(o.w, 0.f);
          } else if (EPI == kEpiResid) {
            const float4 c = *cp;
            o.x += c.x; o.y += c.y; o.z += c.z; o.w += c.w;
          } else if (EPI == kEpiGate) {
            const float4 c = *cp;
            o.x = c.x > 0.f ? o.x : 0.f; o.y = c.y > 0.f ? o.y : 0.f;
            o.z = c.z > 0.f ? o.z : 0.f; o.w = c.w > 0.f ? o.w : 0.f;
          }
          *cp = o;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if (a.planes > 0)  // the map is 3-D
            asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%1, %2, %3}], [%4];"
                         ::"l"(reinterpret_cast<uint64_t>(&cmap)), "r"(cc * 32), "r"(row0), "r"(n),
                         "r"(smem_u32(buf))
                         : "memory");
          else
            asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];"
                         ::"l"(reinterpret_cast<uint64_t>(&cmap)), "r"(x), "r"(row0), "r"(smem_u32(buf))
                         : "memory");
          asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        }
      }
      if (!ok) break;
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
    }
    // every store has left shared memory and landed before the CTA exits
    if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// Weight images: W [N, K] f32 (row-major, [out,in]) -> for each 128-row
// N tile and 64-wide K chunk, a swizzled fp16 hi tile then a lo tile, with
// W scaled by 2^sw. One CTA per (tile, chunk), 256 threads.
// ---------------------------------------------------------------------------
__global__ void k_weight_image(const float* __restrict__ W, int N, int K, float w_scale, uint8_t* __restrict__ out) {
  const int kchunks = K / kBK;
  const int n = blockIdx.x / kchunks, kc = blockIdx.x % kchunks;
  uint8_t* hi = out + size_t(blockIdx.x) * 2 * kTileBytes;
  uint8_t* lo = hi + kTileBytes;
  for (int i = threadIdx.x; i < kBN * kBK; i += blockDim.x) {
    const int r = i / kBK, k = i % kBK;
    const float x = W[size_t(n * kBN + r) * K + kc * kBK + k] * w_scale;
    const __half h = __float2half_rn(x);
    const __half l = __float2half_rn(x - __half2float(h));
    const uint32_t off = swz_offset(r, k);
    *reinterpret_cast<__half*>(hi + off) = h;
    *reinterpret_cast<__half*>(lo + off) = l;
  }
}

// ---------------------------------------------------------------------------
// Host side: the tensor map of an A operand [rows, cols] f32 with row stride
// lda (elements), boxes of [128 rows x 64 cols]. The driver's encoder is
// reached through the runtime's entry-point query, so nothing links libcuda.
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// Returns false if the encoder is unavailable or refuses the map (A must be
// 16-byte aligned and lda a multiple of 4).
// The C operand [rows, cols] f32: boxes of [32 rows x 32 cols], 128-byte swizzle.
inline bool make_c_map(CUtensorMap* map, const float* C, uint64_t rows, uint64_t cols, uint64_t ldc) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (!fn || (reinterpret_cast<uintptr_t>(C) & 15) || (ldc & 3) || cols % 32 || rows == 0) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {ldc * 4};
  const cuuint32_t box[2] = {32, 32};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(C), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The output map of a planes product: [planes, rows, 128] f32, the planes
// contiguous, [1 x 32 x 32] boxes, 128-byte swizzle (as make_c_map per plane).
inline bool make_c_map3(CUtensorMap* map, const float* C, uint64_t rows, uint64_t planes) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (!fn || (reinterpret_cast<uintptr_t>(C) & 15) || rows == 0 || planes == 0) return false;
  const cuuint64_t dims[3] = {128, rows, planes};
  const cuuint64_t strides[2] = {128 * 4, rows * 128 * 4};
  const cuuint32_t box[3] = {32, 32, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(C), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

inline bool make_a_map(CUtensorMap* map, const float* A, uint64_t rows, uint64_t cols, uint64_t lda) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (!fn || (reinterpret_cast<uintptr_t>(A) & 15) || (lda & 3) || cols % kBK || rows == 0) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {lda * 4};
  const cuuint32_t box[2] = {uint32_t(kBK), uint32_t(kBM)};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(A), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace tc
}  // namespace kc
