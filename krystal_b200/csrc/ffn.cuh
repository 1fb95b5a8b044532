// ffn.cuh — the encoder's feed-forward half in one kernel on the tensor
// cores: x += relu(x·W1ᵀ)·W2ᵀ (ffnOracle + addInPlace, oracle.ts:127-139,
// 256-258), with the [rows, F] hidden activations kept on chip.
//
// Same arithmetic as k_tc_gemm<kEpiRelu> followed by k_tc_gemm<kEpiResid>:
// x split at 2^sa into fp16 hi/lo, three MMAs per product into fp32 TMEM,
// h1 = relu(acc · 2^-(sa+sw1)) exactly as the W1 epilogue stores it, then
// split at 2^sa again exactly as the W2 GEMM's split warps split it. So the
// output equals the two-kernel sequence bit for bit, without writing and
// re-reading h1 (3 KB per token and block).
//
// One persistent CTA per SM, 128-row tiles, 320 threads:
//   warp 0     TMA: the x tile (two [128 x 64] f32 boxes) and, per tile,
//              twelve 32 KB weight-image chunks in the order warp 5 consumes
//              them, through a two-stage ring;
//   warps 1-4  split the x tile in place to swizzled fp16 hi | lo;
//   warp 5     MMA issuer. Per tile, for hidden chunks j = 0, 1, 2 of 128
//              columns: P1(j) = x·W1[j]ᵀ into TMEM buffer j % 2, and
//              P2(j) += h1[j]·W2[:, j]ᵀ into the output accumulator, issued
//              P1(0) P1(1) P2(0) P1(2) P2(1) P2(2) so each P1 overlaps the
//              epilogue of the one before;
//   warps 6-9  for each j: TMEM → ×2^-(sa+sw1), ReLU, ×2^sa, split → the
//              fp16 hi | lo operand of P2(j) in shared memory; then the
//              output: TMEM → ×2^-(sa+sw2) + x (TMA-loaded) → TMA store.
// Shared memory: x operand 64 KB, h1 operand 64 KB, weight ring 2 x 32 KB,
// epilogue store buffers 32 KB. TMEM: 512 columns (two 128-column P1
// buffers, one 128-column output accumulator). Every wait is bounded; an
// expired wait sets the error word and the CTA drains and exits.
#pragma once
#include "tc_gemm.cuh"

namespace kc {
namespace tc {

constexpr int kFfnWStages = 2;
constexpr int kFfnChunk = 2 * kTileBytes;                // one weight chunk: hi | lo, 32 KB
constexpr int kFfnXBytes = 2 * kFfnChunk;                // x operand: 2 K-chunks, 64 KB
constexpr int kFfnHBytes = 2 * kFfnChunk;                // h1 operand: 2 K-chunks, 64 KB
constexpr int kFfnSmem = kFfnXBytes + kFfnHBytes + kFfnWStages * kFfnChunk + kEpiBytes + 1024 + 256;
constexpr int kFfnChunksPerTile = 12;                    // 3 x (W1: 2 chunks) + 6 W2 chunks

struct FfnArgs {
  int M;                 // rows
  const uint8_t* w1;     // W1 image [3 n-tiles][2 k-chunks][hi | lo]
  const uint8_t* w2;     // W2 image [1 n-tile][6 k-chunks][hi | lo]
  float a_scale;         // 2^sa, both splits
  float unscale1;        // 2^-(sa + sw1)
  float unscale2;        // 2^-(sa + sw2)
  int* err;
};

// Weight chunk c of a tile, in consumption order: (is_w2, index into its image).
__device__ __forceinline__ const uint8_t* ffn_chunk(const FfnArgs& a, int c) {
  // P1(0): W1 n0 k0,k1 | P1(1): n1 k0,k1 | P2(0): W2 k0,k1 | P1(2): n2 k0,k1 | P2(1): k2,k3 | P2(2): k4,k5
  constexpr int kW2[kFfnChunksPerTile] = {0, 0, 0, 0, 1, 1, 0, 0, 1, 1, 1, 1};
  constexpr int kIdx[kFfnChunksPerTile] = {0, 1, 2, 3, 0, 1, 4, 5, 2, 3, 4, 5};
  return (kW2[c] ? a.w2 : a.w1) + size_t(kIdx[c]) * kFfnChunk;
}

__global__ void __launch_bounds__(kThreadsT, 1) k_tc_ffn(const __grid_constant__ CUtensorMap amap,
                                                          const __grid_constant__ CUtensorMap cmap, FfnArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* xs = smem;                                   // x operand (f32 staging, then hi|lo)
  unsigned char* hs = smem + kFfnXBytes;                      // h1 operand
  unsigned char* ws = hs + kFfnHBytes;                        // weight ring
  float* epi_buf = reinterpret_cast<float*>(ws + kFfnWStages * kFfnChunk);
  uint64_t* bars = reinterpret_cast<uint64_t*>(ws + kFfnWStages * kFfnChunk + kEpiBytes);
  uint64_t* xraw = bars;         // [2] x box landed
  uint64_t* xfull = bars + 2;    // [2] x chunk split
  uint64_t* xempty = bars + 4;   // the tile's P1s are done with x
  uint64_t* wfull = bars + 5;    // [2]
  uint64_t* wempty = bars + 7;   // [2]
  uint64_t* pfull = bars + 9;    // [2] P1 accumulator ready
  uint64_t* pempty = bars + 11;  // [2] P1 accumulator read
  uint64_t* hfull = bars + 13;   // h1 operand written
  uint64_t* hempty = bars + 14;  // P2 done reading the h1 operand
  uint64_t* ofull = bars + 15;   // output accumulator ready
  uint64_t* oempty = bars + 16;  // output accumulator read
  uint64_t* drain = bars + 17;
  uint64_t* cload = bars + 18;   // [4 warps][2 buffers] residual tiles landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 26);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles = (a.M + kBM - 1) / kBM;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; i++) {
      mbar_init(&xraw[i], 1);
      mbar_init(&xfull[i], 128);
      mbar_init(&wfull[i], 1);
      mbar_init(&wempty[i], 1);
      mbar_init(&pfull[i], 1);
      mbar_init(&pempty[i], 128);
    }
    mbar_init(xempty, 1);
    mbar_init(hfull, 128);
    mbar_init(hempty, 1);
    mbar_init(ofull, 1);
    mbar_init(oempty, 128);
    mbar_init(drain, 1);
    for (int i = 0; i < 8; i++) mbar_init(&cload[i], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 5) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t tmem_out = tmem_base + 2 * kBN;

  if (warp == 0) {
    // ---------------- TMA issuer ----------------
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&amap)) : "memory");
      uint32_t it = 0, tl = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, tl++) {
        if (!mbar_wait(xempty, (tl & 1) ^ 1, a.err)) { ok = false; break; }
        for (int kc = 0; kc < 2; kc++) {
          mbar_arrive_expect_tx(&xraw[kc], kFfnChunk);
          tma_load_2d(xs + kc * kFfnChunk, &amap, kc * kBK, t * kBM, &xraw[kc]);
        }
        for (int c = 0; c < kFfnChunksPerTile; c++, it++) {
          const int s = it % kFfnWStages;
          const uint32_t ph = (it / kFfnWStages) & 1;
          if (!mbar_wait(&wempty[s], ph ^ 1, a.err)) { ok = false; break; }
          mbar_arrive_expect_tx(&wfull[s], kFfnChunk);
          const uint8_t* src = ffn_chunk(a, c);
          bulk_g2s(ws + s * kFfnChunk, src, kTileBytes, &wfull[s]);
          bulk_g2s(ws + s * kFfnChunk + kTileBytes, src + kTileBytes, kTileBytes, &wfull[s]);
        }
      }
      // every copy issued lands before the CTA may exit
      for (uint32_t j = it > uint32_t(kFfnWStages) ? it - kFfnWStages : 0u; j < it; j++)
        mbar_wait(&wfull[j % kFfnWStages], (j / kFfnWStages) & 1, a.err);
      if (tl > 0)
        for (int kc = 0; kc < 2; kc++) mbar_wait(&xraw[kc], (tl - 1) & 1, a.err);
    }
    __syncwarp();
  } else if (warp <= 4) {
    // ---------------- split the x tile: f32 staging -> swizzled fp16 hi / lo ----------------
    const int tid = threadIdx.x - 32;
    uint32_t tl = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, tl++) {
      bool ok = true;
      for (int kc = 0; kc < 2; kc++) {
        const int mine = mbar_wait(&xraw[kc], tl & 1, a.err) ? 1 : 0;
        int all;
        asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %1, 0;\n\t"
                     "bar.red.and.pred p, 1, 128, p;\n\tselp.u32 %0, 1, 0, p;\n\t}"
                     : "=r"(all) : "r"(mine) : "memory");
        if (!all) { ok = false; break; }
        unsigned char* st = xs + kc * kFfnChunk;
        float4 v[16];
        const float4* stage = reinterpret_cast<const float4*>(st);
#pragma unroll
        for (int i = 0; i < 16; i++) v[i] = stage[i * 128 + tid];
        asm volatile("bar.sync 1, 128;" ::: "memory");
        bool bad = false;
#pragma unroll
        for (int i = 0; i < 16; i++) {
          const int L = i * 128 + tid;
          const int r = L >> 4, c4 = L & 15;
          float xv[4] = {v[i].x * a.a_scale, v[i].y * a.a_scale, v[i].z * a.a_scale, v[i].w * a.a_scale};
          float hi[4], lo[4];
#pragma unroll
          for (int e = 0; e < 4; e++) {
            bad |= !(fabsf(xv[e]) < 32768.0f);
            split_f32(xv[e], hi[e], lo[e]);
          }
          const uint32_t off = swz_offset(r, c4 * 4);
          *reinterpret_cast<uint2*>(st + off) =
              make_uint2(h2u(__floats2half2_rn(hi[0], hi[1])), h2u(__floats2half2_rn(hi[2], hi[3])));
          *reinterpret_cast<uint2*>(st + kTileBytes + off) =
              make_uint2(h2u(__floats2half2_rn(lo[0], lo[1])), h2u(__floats2half2_rn(lo[2], lo[3])));
        }
        if (bad) atomicOr(a.err, kErrOverflow);
        fence_proxy_async_smem();
        mbar_arrive(&xfull[kc]);
      }
      if (!ok) break;
    }
  } else if (warp == 5) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      uint32_t it = 0, tl = 0;
      bool ok = true;
      // three MMAs per 16-wide K step over one 64-wide chunk pair (A, B)
      auto chunk_mma = [&](uint32_t d, uint32_t a_saddr, uint32_t b_saddr, bool first) {
#pragma unroll
        for (int kk = 0; kk < kBK / 16; kk++) {
          const uint64_t ah = smem_desc(a_saddr + kk * 32), al = smem_desc(a_saddr + kTileBytes + kk * 32);
          const uint64_t bh = smem_desc(b_saddr + kk * 32), bl = smem_desc(b_saddr + kTileBytes + kk * 32);
          mma_f16(d, ah, bh, (first && kk == 0) ? 0u : 1u);
          mma_f16(d, ah, bl, 1u);
          mma_f16(d, al, bh, 1u);
        }
      };
      auto next_w = [&](uint32_t& s_out) -> bool {  // the next weight chunk has landed
        const int s = it % kFfnWStages;
        const uint32_t ph = (it / kFfnWStages) & 1;
        if (!mbar_wait(&wfull[s], ph, a.err)) return false;
        tc_fence_after();
        s_out = smem_u32(ws + s * kFfnChunk);
        return true;
      };
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, tl++) {
        for (int kc = 0; kc < 2 && ok; kc++) ok = mbar_wait(&xfull[kc], tl & 1, a.err);
        if (!ok) break;
        tc_fence_after();
        // the schedule P1(0) P1(1) P2(0) P1(2) P2(1) P2(2): step -> (is P2, hidden chunk j)
        constexpr int kP2[6] = {0, 0, 1, 0, 1, 1};
        constexpr int kJ[6] = {0, 1, 0, 2, 1, 2};
        for (int step = 0; step < 6 && ok; step++) {
          const bool p2 = kP2[step] != 0;
          const int j = kJ[step];
          const uint32_t u = 3 * tl + j;
          if (!p2) {
            const uint32_t buf = u & 1;
            if (!mbar_wait(&pempty[buf], ((u >> 1) & 1) ^ 1, a.err)) { ok = false; break; }
            tc_fence_after();
            for (int kc = 0; kc < 2; kc++, it++) {
              uint32_t sb;
              if (!next_w(sb)) { ok = false; break; }
              chunk_mma(tmem_base + buf * kBN, smem_u32(xs + kc * kFfnChunk), sb, kc == 0);
              mma_commit(&wempty[it % kFfnWStages]);
            }
            if (!ok) break;
            mma_commit(&pfull[buf]);
            if (j == 2) mma_commit(xempty);
          } else {
            if (j == 0 && !mbar_wait(oempty, (tl & 1) ^ 1, a.err)) { ok = false; break; }
            if (!mbar_wait(hfull, u & 1, a.err)) { ok = false; break; }
            tc_fence_after();
            for (int kc = 0; kc < 2; kc++, it++) {
              uint32_t sb;
              if (!next_w(sb)) { ok = false; break; }
              chunk_mma(tmem_out, smem_u32(hs + kc * kFfnChunk), sb, j == 0 && kc == 0);
              mma_commit(&wempty[it % kFfnWStages]);
            }
            if (!ok) break;
            mma_commit(hempty);
            if (j == 2) mma_commit(ofull);
          }
        }
      }
      // every MMA this thread issued completes before TMEM is released
      mma_commit(drain);
      mbar_wait(drain, 0, a.err);
    }
    __syncwarp();
  } else {
    // ---------------- epilogue ----------------
    const int g = warp & 3;  // TMEM lane quarter this warp may read
    const int ew = warp - 6;
    unsigned char* bufs = reinterpret_cast<unsigned char*>(epi_buf) + ew * 2 * kEpiBuf;
    uint32_t cphase = 0;
    uint32_t tl = 0;
    bool ok = true;
    const int row = g * 32 + lane;  // this lane's row of the tile
    for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, tl++) {
      // h1 for hidden chunks j = 0, 1, 2: the operand of P2(j)
      for (int j = 0; j < 3 && ok; j++) {
        const uint32_t u = 3 * tl + j, buf = u & 1;
        int okw = 0;
        if (lane == 0)
          okw = (mbar_wait(&pfull[buf], (u >> 1) & 1, a.err) && mbar_wait(hempty, (u & 1) ^ 1, a.err)) ? 1 : 0;
        okw = __shfl_sync(0xffffffffu, okw, 0);
        if (!okw) { ok = false; break; }
        tc_fence_after();
        bool bad = false;
#pragma unroll 1
        for (int cg = 0; cg < kBN / 32; cg++) {
          float v[32];
          tmem_ld32(tmem_base + (uint32_t(g * 32) << 16) + buf * kBN + cg * 32, v);
          // columns cg*32 .. +31 of this 128-column chunk: K chunk cg / 2, K offset (cg % 2) * 32
          unsigned char* base = hs + (cg >> 1) * kFfnChunk;
#pragma unroll
          for (int q = 0; q < 4; q++) {  // 8 columns per 16-byte store
            uint32_t hw[4], lw[4];
#pragma unroll
            for (int e = 0; e < 4; e++) {
              float h2[2], l2[2];
#pragma unroll
              for (int z = 0; z < 2; z++) {
                const float y = fmaxf(v[8 * q + 2 * e + z] * a.unscale1, 0.f) * a.a_scale;
                bad |= !(fabsf(y) < 32768.0f);
                split_f32(y, h2[z], l2[z]);
              }
              hw[e] = h2u(__floats2half2_rn(h2[0], h2[1]));
              lw[e] = h2u(__floats2half2_rn(l2[0], l2[1]));
            }
            const uint32_t off = swz_offset(row, (cg & 1) * 32 + 8 * q);
            *reinterpret_cast<uint4*>(base + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
            *reinterpret_cast<uint4*>(base + kTileBytes + off) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
          }
        }
        if (bad) atomicOr(a.err, kErrOverflow);
        tc_fence_before();
        mbar_arrive(&pempty[buf]);
        fence_proxy_async_smem();
        mbar_arrive(hfull);
      }
      if (!ok) break;
      // the output: x += acc · 2^-(sa+sw2), through 128-byte swizzled 32x32 blocks
      int okw = 0;
      if (lane == 0) okw = mbar_wait(ofull, tl & 1, a.err) ? 1 : 0;
      okw = __shfl_sync(0xffffffffu, okw, 0);
      if (!okw) { ok = false; break; }
      tc_fence_after();
      const int row0 = t * kBM + g * 32;
#pragma unroll 1
      for (int cc = 0; cc < kBN / 32; cc++) {
        const int b = cc & 1;
        unsigned char* eb = bufs + b * kEpiBuf;
        const int x = cc * 32;
        if (lane == 0) {
          asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
          mbar_arrive_expect_tx(&cload[ew * 2 + b], kEpiBuf);
          asm volatile(
              "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
              ::"r"(smem_u32(eb)), "l"(reinterpret_cast<uint64_t>(&cmap)), "r"(x), "r"(row0),
              "r"(smem_u32(&cload[ew * 2 + b]))
              : "memory");
        }
        float v[32];
        tmem_ld32(tmem_out + (uint32_t(g * 32) << 16) + cc * 32, v);
        const bool mine = mbar_wait(&cload[ew * 2 + b], (cphase >> b) & 1, a.err);
        cphase ^= 1u << b;
        if (!__all_sync(0xffffffffu, mine)) { ok = false; break; }
        unsigned char* rowp = eb + lane * 128;
#pragma unroll
        for (int jj = 0; jj < 8; jj++) {
          float4* cp = reinterpret_cast<float4*>(rowp + ((jj ^ (lane & 7)) << 4));
          const float4 c = *cp;
          float4 o = make_float4(v[4 * jj] * a.unscale2, v[4 * jj + 1] * a.unscale2, v[4 * jj + 2] * a.unscale2,
                                 v[4 * jj + 3] * a.unscale2);
          o.x += c.x; o.y += c.y; o.z += c.z; o.w += c.w;
          *cp = o;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];"
                       ::"l"(reinterpret_cast<uint64_t>(&cmap)), "r"(x), "r"(row0), "r"(smem_u32(eb))
                       : "memory");
          asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        }
      }
      if (!ok) break;
      tc_fence_before();
      mbar_arrive(oempty);
    }
    if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

}  // namespace tc
}  // namespace kc
