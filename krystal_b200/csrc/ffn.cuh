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
//   warp 0     TMA: lane 0 the twelve 32 KB weight-image chunks per tile
//              (W1 then W2) through a three-stage ring; lane 1 the x tile
//              (two [128 x 64] f32 boxes) as soon as the previous tile's P1
//              products release the operand;
//   warps 1-4  split the x tile in place to swizzled fp16 hi | lo, and
//              share the epilogues below with warps 6-9;
//   warp 5     MMA issuer. Per tile: P1(j) = x·W1[j]ᵀ for hidden chunks
//              j = 0, 1, 2 of 128 columns into TMEM buffer j (A and B in
//              shared memory), then P2(j) += h1[j]·W2[:, j]ᵀ into the output
//              accumulator with A = h1[j] read from TMEM buffer j itself;
//   epilogues  for each j: TMEM → ×2^-(sa+sw1), ReLU, ×2^sa, split → fp16
//              hi | lo written back over the same TMEM columns (each 16-column
//              K step: 8 columns of hi pairs, then 8 of lo pairs); then the
//              output: TMEM → ×2^-(sa+sw2) + x → TMA store, with x prefetched
//              into shared memory a tile ahead. Warps 6-9 take hidden columns
//              0-63 of each chunk and output columns 0-63; warps 1-4 the
//              other halves, and they split the next tile's x before their
//              output half.
// Keeping h1 in TMEM halves the shared-memory reads of the W2 products and
// removes the h1 stores: the SS products at N = 128 alone read shared memory
// at its full rate. Shared memory: x operand 64 KB, output staging 8 warps x
// 2 x 4 KB, weight ring 3 x 32 KB. TMEM: 512 columns (three 128-column P1 /
// h1 buffers, one 128-column output accumulator). Every wait is bounded; an
// expired wait sets the error word and the CTA drains and exits.
#pragma once
#include "tc_gemm.cuh"

namespace kc {
namespace tc {

constexpr int kFfnWStages = 3;
constexpr int kFfnChunk = 2 * kTileBytes;                // one weight chunk: hi | lo, 32 KB
constexpr int kFfnXBytes = 2 * kFfnChunk;                // x operand: 2 K-chunks, 64 KB
constexpr int kFfnEBytes = 8 * 2 * kEpiBuf;              // output staging: 8 warps x 2 blocks, 64 KB
constexpr int kFfnSmem = kFfnXBytes + kFfnEBytes + kFfnWStages * kFfnChunk + 1024 + 512;
constexpr int kFfnChunksPerTile = 12;                    // W1: 3 n-tiles x 2 k-chunks, then W2: 6 k-chunks

struct FfnArgs {
  int M;                 // rows
  const uint8_t* w1;     // W1 image [3 n-tiles][2 k-chunks][hi | lo]
  const uint8_t* w2;     // W2 image [1 n-tile][6 k-chunks][hi | lo]
  float a_scale;         // 2^sa, both splits
  float unscale1;        // 2^-(sa + sw1)
  float unscale2;        // 2^-(sa + sw2)
  int* err;
  int inject_expiry;  // test hook: the producers report an expired wait before they issue any copy
};

// Weight chunk c of a tile, in consumption order: P1(0..2) take W1 chunks
// 0..5, P2(0..2) take W2 chunks 0..5.
__device__ __forceinline__ const uint8_t* ffn_chunk(const FfnArgs& a, int c) {
  return c < 6 ? a.w1 + size_t(c) * kFfnChunk : a.w2 + size_t(c - 6) * kFfnChunk;
}

__global__ void __launch_bounds__(kThreadsT, 1) k_tc_ffn(const __grid_constant__ CUtensorMap amap,
                                                          const __grid_constant__ CUtensorMap cmap, FfnArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* xs = smem;                                   // x operand (f32 staging, then hi|lo)
  unsigned char* es = smem + kFfnXBytes;                      // output staging
  unsigned char* ws = es + kFfnEBytes;                        // weight ring
  uint64_t* bars = reinterpret_cast<uint64_t*>(ws + kFfnWStages * kFfnChunk);
  uint64_t* xraw = bars;         // [2] x box landed
  uint64_t* xfull = bars + 2;    // [2] x chunk split
  uint64_t* xempty = bars + 4;   // the tile's P1s are done with x
  uint64_t* wfull = bars + 5;    // [kFfnWStages]
  uint64_t* wempty = bars + 8;   // [kFfnWStages]
  uint64_t* pfull = bars + 11;   // [3] P1 accumulator j ready
  uint64_t* pempty = bars + 14;  // [3] P2(j) done reading h1 from buffer j
  uint64_t* hfull = bars + 17;   // [3] h1 chunk j written to TMEM
  uint64_t* ofull = bars + 20;   // output accumulator ready
  uint64_t* oempty = bars + 21;  // output accumulator read
  uint64_t* drain = bars + 22;
  uint64_t* cload = bars + 23;   // [8 epilogue warps][2 blocks] residual landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 39);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles = (a.M + kBM - 1) / kBM;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; i++) {
      mbar_init(&xraw[i], 1);
      mbar_init(&xfull[i], 128);
    }
    for (int i = 0; i < 3; i++) {
      mbar_init(&pfull[i], 1);
      mbar_init(&pempty[i], 1);
      mbar_init(&hfull[i], 256);
    }
    for (int i = 0; i < kFfnWStages; i++) {
      mbar_init(&wfull[i], 1);
      mbar_init(&wempty[i], 1);
    }
    mbar_init(xempty, 1);
    mbar_init(ofull, 1);
    mbar_init(oempty, 256);
    mbar_init(drain, 1);
    for (int i = 0; i < 16; i++) mbar_init(&cload[i], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 5) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t tmem_out = tmem_base + 3 * kBN;

  if (warp == 0) {
    // ---------------- TMA issuers ----------------
    // lane 0 streams the weight chunks; lane 1 loads each tile's x as soon as
    // the previous tile's P1 products release it (not behind the W2 chunks)
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      if (a.inject_expiry) {  // as if the first wait had expired: nothing is issued
        atomicOr(a.err, kErrTimeout);
        ok = false;
      }
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
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
        mbar_wait_drain(&wfull[j % kFfnWStages], (j / kFfnWStages) & 1);
    } else if (lane == 1) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&amap)) : "memory");
      uint32_t tl = 0;
      for (int t = blockIdx.x; t < tiles && !a.inject_expiry; t += gridDim.x, tl++) {
        if (!mbar_wait(xempty, (tl & 1) ^ 1, a.err)) break;
        for (int kc = 0; kc < 2; kc++) {
          mbar_arrive_expect_tx(&xraw[kc], kFfnChunk);
          tma_load_2d(xs + kc * kFfnChunk, &amap, kc * kBK, t * kBM, &xraw[kc]);
        }
      }
      // the last x issued lands before the CTA may exit
      if (tl > 0)
        for (int kc = 0; kc < 2; kc++) mbar_wait_drain(&xraw[kc], (tl - 1) & 1);
    }
    __syncwarp();
  } else if (warp == 5) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      uint32_t it = 0, tl = 0;
      bool ok = true;
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
        // P1(j): three MMAs per 16-wide K step, A = x (shared), B = W1 chunk
        for (int j = 0; j < 3 && ok; j++) {
          const uint32_t d = tmem_base + j * kBN;
          if (!mbar_wait(&pempty[j], (tl & 1) ^ 1, a.err)) { ok = false; break; }
          tc_fence_after();
          for (int kc = 0; kc < 2; kc++, it++) {
            uint32_t sb;
            if (!next_w(sb)) { ok = false; break; }
            const uint32_t sa = smem_u32(xs + kc * kFfnChunk);
#pragma unroll
            for (int kk = 0; kk < kBK / 16; kk++) {
              const uint64_t ah = smem_desc(sa + kk * 32), al = smem_desc(sa + kTileBytes + kk * 32);
              const uint64_t bh = smem_desc(sb + kk * 32), bl = smem_desc(sb + kTileBytes + kk * 32);
              mma_f16(d, ah, bh, (kc == 0 && kk == 0) ? 0u : 1u);
              mma_f16(d, ah, bl, 1u);
              mma_f16(d, al, bh, 1u);
            }
            mma_commit(&wempty[it % kFfnWStages]);
          }
          if (!ok) break;
          mma_commit(&pfull[j]);
        }
        if (!ok) break;
        mma_commit(xempty);
        // P2(j): A = h1 chunk j in TMEM buffer j, B = W2 chunk
        for (int j = 0; j < 3 && ok; j++) {
          if (j == 0 && !mbar_wait(oempty, (tl & 1) ^ 1, a.err)) { ok = false; break; }
          if (!mbar_wait(&hfull[j], tl & 1, a.err)) { ok = false; break; }
          tc_fence_after();
          for (int kc = 0; kc < 2; kc++, it++) {
            uint32_t sb;
            if (!next_w(sb)) { ok = false; break; }
#pragma unroll
            for (int kk = 0; kk < kBK / 16; kk++) {
              const uint32_t ah = tmem_base + j * kBN + kc * 64 + kk * 16, al = ah + 8;
              const uint64_t bh = smem_desc(sb + kk * 32), bl = smem_desc(sb + kTileBytes + kk * 32);
              mma_f16_ts(tmem_out, ah, bh, (j == 0 && kc == 0 && kk == 0) ? 0u : 1u);
              mma_f16_ts(tmem_out, ah, bl, 1u);
              mma_f16_ts(tmem_out, al, bh, 1u);
            }
            mma_commit(&wempty[it % kFfnWStages]);
          }
          if (!ok) break;
          mma_commit(&pempty[j]);
        }
        if (!ok) break;
        mma_commit(ofull);
      }
      // every MMA this thread issued completes before TMEM is released
      mma_commit(drain);
      mbar_wait_drain(drain, 0);
    }
    __syncwarp();
  } else {
    // ---------------- split (warps 1-4) and the epilogues (warps 1-4, 6-9) ----------------
    const bool helper = warp <= 4;
    const int half = helper ? 1 : 0;             // which 64 columns of each 128-column block
    const int wi = helper ? warp - 1 + 4 : warp - 6;  // epilogue buffer / barrier index 0..7
    const int q = warp & 3;                      // TMEM lane quarter this warp may read
    unsigned char* eb[2] = {es + wi * 2 * kEpiBuf, es + wi * 2 * kEpiBuf + kEpiBuf};
    // the x tile of tile number tl: f32 staging -> swizzled fp16 hi / lo, in place
    auto split = [&](uint32_t tl) -> bool {
      const int tid = threadIdx.x - 32;
      for (int kc = 0; kc < 2; kc++) {
        const int mine = mbar_wait(&xraw[kc], tl & 1, a.err) ? 1 : 0;
        int all;
        asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %1, 0;\n\t"
                     "bar.red.and.pred p, 1, 128, p;\n\tselp.u32 %0, 1, 0, p;\n\t}"
                     : "=r"(all) : "r"(mine) : "memory");
        if (!all) return false;
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
      return true;
    };
    // 32 columns (two K steps) of a P1 accumulator -> ReLU, re-split, packed
    // for the TMEM A operand: per K step, hi pairs then lo pairs
    auto pack_h = [&](const float* v, uint32_t* w, bool& bad) {
#pragma unroll
      for (int ks = 0; ks < 2; ks++)
#pragma unroll
        for (int e = 0; e < 8; e++) {
          float h2[2], l2[2];
#pragma unroll
          for (int z = 0; z < 2; z++) {
            const float y = fmaxf(v[16 * ks + 2 * e + z] * a.unscale1, 0.f) * a.a_scale;
            bad |= !(fabsf(y) < 32768.0f);
            split_f32(y, h2[z], l2[z]);
          }
          w[16 * ks + e] = h2u(__floats2half2_rn(h2[0], h2[1]));
          w[16 * ks + 8 + e] = h2u(__floats2half2_rn(l2[0], l2[1]));
        }
    };
    // this warp's 64 columns of hidden chunk j of tile number tl, in place in TMEM
    auto e1 = [&](uint32_t tl, int j) -> bool {
      int okw = 0;
      if (lane == 0) okw = mbar_wait(&pfull[j], tl & 1, a.err) ? 1 : 0;
      okw = __shfl_sync(0xffffffffu, okw, 0);
      if (!okw) return false;
      tc_fence_after();
      const uint32_t ta = tmem_base + (uint32_t(q * 32) << 16) + j * kBN + half * 64;
      float v0[32], v1[32];
      uint32_t w[32];
      bool bad = false;
      tmem_ld32(ta, v0);
      tmem_ld32_async(ta + 32, v1);  // in flight while the first 32 columns convert
      pack_h(v0, w, bad);
      tmem_st32(ta, w);
      tmem_ld_wait(v1);
      pack_h(v1, w, bad);
      tmem_st32(ta + 32, w);
      tmem_st_wait();
      if (bad) atomicOr(a.err, kErrOverflow);
      tc_fence_before();
      mbar_arrive(&hfull[j]);
      return true;
    };
    // the residual x rows of tile t for this warp's output blocks, into staging
    auto prefetch = [&](int t) {
      if (lane == 0) {
        asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");  // staging free again
        for (int b = 0; b < 2; b++) {
          mbar_arrive_expect_tx(&cload[wi * 2 + b], kEpiBuf);
          asm volatile(
              "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
              ::"r"(smem_u32(eb[b])), "l"(reinterpret_cast<uint64_t>(&cmap)), "r"((half * 2 + b) * 32),
              "r"(t * kBM + q * 32), "r"(smem_u32(&cload[wi * 2 + b]))
              : "memory");
        }
      }
      __syncwarp();
    };
    // this warp's half of the output of tile t (number tl): x += acc · 2^-(sa+sw2)
    auto e2 = [&](uint32_t tl, int t) -> bool {
      int okw = 0;
      if (lane == 0) okw = mbar_wait(ofull, tl & 1, a.err) ? 1 : 0;
      okw = __shfl_sync(0xffffffffu, okw, 0);
      if (!okw) return false;
      tc_fence_after();
      float v[2][32];
      tmem_ld32(tmem_out + (uint32_t(q * 32) << 16) + half * 64, v[0]);
      tmem_ld32_async(tmem_out + (uint32_t(q * 32) << 16) + half * 64 + 32, v[1]);
      tmem_ld_wait(v[1]);
      tc_fence_before();
      mbar_arrive(oempty);  // the accumulator is free for the next tile
#pragma unroll
      for (int b = 0; b < 2; b++) {
        const bool mine = mbar_wait(&cload[wi * 2 + b], tl & 1, a.err);
        if (!__all_sync(0xffffffffu, mine)) return false;
        unsigned char* rowp = eb[b] + lane * 128;
#pragma unroll
        for (int jj = 0; jj < 8; jj++) {
          float4* cp = reinterpret_cast<float4*>(rowp + ((jj ^ (lane & 7)) << 4));
          const float4 c = *cp;
          float4 o = make_float4(v[b][4 * jj] * a.unscale2, v[b][4 * jj + 1] * a.unscale2,
                                 v[b][4 * jj + 2] * a.unscale2, v[b][4 * jj + 3] * a.unscale2);
          o.x += c.x; o.y += c.y; o.z += c.z; o.w += c.w;
          *cp = o;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];"
                       ::"l"(reinterpret_cast<uint64_t>(&cmap)), "r"((half * 2 + b) * 32), "r"(t * kBM + q * 32),
                       "r"(smem_u32(eb[b]))
                       : "memory");
          asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        }
      }
      return true;
    };
    bool ok = true;
    uint32_t tl = 0;
    int pending = -1;  // tile number whose residual prefetch is in flight
    if (blockIdx.x < tiles) {
      prefetch(blockIdx.x);
      pending = 0;
    }
    if (helper && blockIdx.x < tiles) ok = split(0);
    for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, tl++) {
      for (int j = 0; j < 3 && ok; j++) ok = e1(tl, j);
      if (ok && helper && t + int(gridDim.x) < tiles) ok = split(tl + 1);
      if (ok) ok = e2(tl, t);
      if (ok) pending = -1;
      if (ok && t + int(gridDim.x) < tiles) {
        prefetch(t + gridDim.x);
        pending = int(tl + 1);
      }
    }
    // a residual prefetch left unconsumed by an error lands before the CTA exits
    if (pending >= 0 && lane == 0)
      for (int b = 0; b < 2; b++) mbar_wait_drain(&cload[wi * 2 + b], uint32_t(pending) & 1);
    // every store has left shared memory and landed before the CTA exits
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
