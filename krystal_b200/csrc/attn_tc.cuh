// attn_tc.cuh — the encoder's attention half in one kernel: the q|k|v
// projection on the tensor cores, record-local attention and the residual
// add (attentionOracle in local mode + addInPlace, forward/oracle.ts:64-105,
// 250-256), with q, k and v never leaving the SM.
//
// Same arithmetic as k_tc_gemm<kEpiStore> (qkv = x·Wqkvᵀ) followed by
// k_local_attn_fast, bit for bit: x split at 2^sa into fp16 hi / lo, three
// MMAs per 16-wide K step into fp32 TMEM in the GEMM's order, q|k|v =
// acc · 2^-(sa+sw) in f32, then per (token, head) the same fmaf chains for the
// scores, the same softmax and the same p·v order, and x += o.
//
// Tiles are record-aligned row ranges: tile k owns the records whose first
// row lies in [120k, 120k + 120). A record has at most 8 rows, so the owned
// rows [a_k, a_(k+1)) number at most 127 and the 128-row MMA block loaded from
// a_k holds every row any owned token attends to; rows past the owned range
// are computed and dropped.
//
// One persistent CTA per SM, 384 threads:
//   warp 0      TMA: the x block (four [128 x 32] f32 boxes, 128-byte
//               swizzled) and the six 32 KB Wqkv image chunks per tile
//               through a three-stage ring;
//   warp 1      MMA issuer: q into TMEM buffer tile % 2 (columns 0 or 384),
//               then k (128) and v (256) once the previous tile has staged
//               its k and v;
//   warps 2-3   split the x block in place to fp16 hi | lo (each row's
//               bytes only, so every warp works on its own rows);
//   warps 4-11  epilogue, two halves of four warps (one per TMEM lane
//               quarter); half h takes heads 2h and 2h+1, one per round:
//               stage the head's k | v rows in shared memory, one thread per
//               token computes its scores, softmax and output, writes the
//               output over its own staged k row, and the warps add the
//               residual with coalesced row loads and stores.
// Shared memory: x operand 64 KB, weight ring 3 x 32 KB, k|v staging 2 x 32
// KB. TMEM: 512 columns. Every wait is bounded; an expired wait sets the
// error word and the CTA drains and exits.
#pragma once
#include "common.cuh"
#include "tc_gemm.cuh"

namespace kc {
namespace tc {

constexpr int kAtWindow = 120;
constexpr int kAtThreads = 384;
constexpr int kAtChunk = 2 * kTileBytes;                 // one weight chunk / x K-chunk: 32 KB
constexpr int kAtXBytes = 2 * kAtChunk;                  // x operand, 64 KB
constexpr int kAtWStages = 2;
constexpr int kAtSlotBytes = 128 * 256;                  // one head's k | v for 128 rows
constexpr int kAtResBytes = 128 * 128;                   // one head's 32 columns of x for 128 rows
constexpr int kAtSmem = kAtXBytes + kAtWStages * kAtChunk + 2 * kAtSlotBytes + 2 * kAtResBytes + 1024 + 512;

struct AttnTcArgs {
  int T;                       // rows (compact tokens)
  int tiles;                   // ceil(T / kAtWindow)
  const int* tile_row;         // [tiles + 1]: first row of each tile, T last (k_attn_tiles)
  const uint32_t* row_rc;      // [T]: position in the record << 4 | record row count
  const uint8_t* w;            // Wqkv image [3 n-tiles][2 k-chunks][hi | lo]
  float a_scale;               // 2^sa
  float unscale;               // 2^-(sa + sw)
  float* x;                    // [T, 128], updated in place
  const uint32_t* tok_recpos;  // [T]: record << 3 | position
  const uint32_t* word_ids;    // optional [records * 8]: the same-word bias's labels
  float word_alpha;
  float scale;                 // 1/sqrt(head dim)
  int* err;
  int inject_expiry;           // test hook: the producer reports an expired wait before it issues any copy
};

// Per batch, shared by every encoder block: per row its position in its
// record and the record's row count, and per tile its first row — the first
// record start at or after row 120k (T past the end). One thread per row.
__global__ void k_attn_tiles(const uint32_t* __restrict__ tok_recpos, const uint32_t* __restrict__ rec_start,
                             const uint2* __restrict__ rec_meta, int T, int tiles, uint32_t* __restrict__ row_rc,
                             int* __restrict__ tile_row) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r == 0) tile_row[tiles] = T;
  if (r >= T) return;
  const uint32_t g = tok_recpos[r] >> 3;
  const uint32_t s = rec_start[g], cnt = rec_meta[g].y & 15u;
  row_rc[r] = ((uint32_t(r) - s) << 4) | cnt;
  if (r % kAtWindow == 0) tile_row[r / kAtWindow] = s == uint32_t(r) ? r : int(s + cnt);
}

__device__ __forceinline__ void named_bar(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

// k | v staging: row i of a slot is 16 float4 (k 0-7, v 8-15), float4 f at f ^ (i & 15)
__device__ __forceinline__ float4* at_row(unsigned char* slot, int i) {
  return reinterpret_cast<float4*>(slot + i * 256);
}

// Row i of a slot as one shared address with the row's swizzle in bits 4-7:
// float4 f of the row is at (at_key(slot, i) ^ (f << 4)).
__device__ __forceinline__ uint32_t at_key(uint32_t slot_u32, int i) { return slot_u32 + i * 256 + ((i & 15) << 4); }

// A shared float4 where p holds, zeros elsewhere (no load issued).
__device__ __forceinline__ float4 lds4_if(uint32_t addr, bool p) {
  float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
  asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %5, 0;\n\t@q ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];\n\t}"
               : "+f"(v.x), "+f"(v.y), "+f"(v.z), "+f"(v.w)
               : "r"(addr), "r"(int(p)));
  return v;
}

// WORDS: the same-word bias is on (a.word_ids set); the kernel without it
// keeps no per-key word registers.
template <bool WORDS>
__global__ void __launch_bounds__(kAtThreads, 1) k_tc_attn(const __grid_constant__ CUtensorMap xmap, AttnTcArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* xs = smem;                                   // x operand (f32 boxes, then hi|lo)
  unsigned char* ws = smem + kAtXBytes;                       // weight ring
  unsigned char* kvs = ws + kAtWStages * kAtChunk;            // k|v staging, two slots
  unsigned char* res = kvs + 2 * kAtSlotBytes;                // residual x columns, one per half
  uint64_t* bars = reinterpret_cast<uint64_t*>(res + 2 * kAtResBytes);
  uint64_t* xraw = bars;         // [2] x K-chunk landed
  uint64_t* xfull = bars + 2;    // [2] x K-chunk split
  uint64_t* xempty = bars + 4;   // the tile's MMAs are done with x
  uint64_t* wfull = bars + 5;    // [kAtWStages]
  uint64_t* wempty = bars + 8;   // [kAtWStages]
  uint64_t* accfull = bars + 11; // q, k, v of the tile ready
  uint64_t* qempty = bars + 12;  // [2] q buffer read
  uint64_t* kvempty = bars + 14; // k and v read
  uint64_t* drain = bars + 15;
  uint64_t* rfull = bars + 16;   // [2] a half's residual columns landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 18);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; i++) {
      mbar_init(&xraw[i], 1);
      mbar_init(&xfull[i], 64);
      mbar_init(&qempty[i], 256);
    }
    for (int i = 0; i < kAtWStages; i++) {
      mbar_init(&wfull[i], 1);
      mbar_init(&wempty[i], 1);
    }
    mbar_init(xempty, 1);
    mbar_init(accfull, 1);
    mbar_init(kvempty, 256);
    mbar_init(drain, 1);
    mbar_init(&rfull[0], 1);
    mbar_init(&rfull[1], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA issuer ----------------
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&xmap)) : "memory");
      uint32_t it = 0, tl = 0;
      bool ok = true;
      if (a.inject_expiry) {  // as if the first wait had expired: nothing is issued
        atomicOr(a.err, kErrTimeout);
        ok = false;
      }
      for (int k = blockIdx.x; k < a.tiles && ok; k += gridDim.x, tl++) {
        const int row0 = a.tile_row[k];
        if (!mbar_wait(xempty, (tl & 1) ^ 1, a.err)) { ok = false; break; }
        for (int kc = 0; kc < 2; kc++) {
          mbar_arrive_expect_tx(&xraw[kc], kAtChunk);
          for (int b = 0; b < 2; b++)
            tma_load_2d(xs + kc * kAtChunk + b * kTileBytes, &xmap, kc * 64 + b * 32, row0, &xraw[kc]);
        }
        for (int c = 0; c < 6; c++, it++) {
          const int s = it % kAtWStages;
          const uint32_t ph = (it / kAtWStages) & 1;
          if (!mbar_wait(&wempty[s], ph ^ 1, a.err)) { ok = false; break; }
          mbar_arrive_expect_tx(&wfull[s], kAtChunk);
          const uint8_t* src = a.w + size_t(c) * kAtChunk;
          bulk_g2s(ws + s * kAtChunk, src, kTileBytes, &wfull[s]);
          bulk_g2s(ws + s * kAtChunk + kTileBytes, src + kTileBytes, kTileBytes, &wfull[s]);
        }
      }
      // every copy issued lands before the CTA may exit
      for (uint32_t j = it > uint32_t(kAtWStages) ? it - kAtWStages : 0u; j < it; j++)
        mbar_wait_drain(&wfull[j % kAtWStages], (j / kAtWStages) & 1);
      if (tl > 0)
        for (int kc = 0; kc < 2; kc++) mbar_wait_drain(&xraw[kc], (tl - 1) & 1);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      uint32_t it = 0, tl = 0;
      bool ok = true;
      for (int k = blockIdx.x; k < a.tiles && ok; k += gridDim.x, tl++) {
        for (int kc = 0; kc < 2 && ok; kc++) ok = mbar_wait(&xfull[kc], tl & 1, a.err);
        if (!ok) break;
        const uint32_t qb = tl & 1;
        if (!mbar_wait(&qempty[qb], ((tl >> 1) & 1) ^ 1, a.err)) { ok = false; break; }
        tc_fence_after();
        for (int n = 0; n < 3 && ok; n++) {
          if (n == 1) {  // k and v overwrite the previous tile's once it has staged them
            if (!mbar_wait(kvempty, (tl & 1) ^ 1, a.err)) { ok = false; break; }
            tc_fence_after();
          }
          const uint32_t d = tmem_base + (n == 0 ? (qb ? 384u : 0u) : uint32_t(128 * n));
          for (int kc = 0; kc < 2; kc++, it++) {
            const int s = it % kAtWStages;
            if (!mbar_wait(&wfull[s], (it / kAtWStages) & 1, a.err)) { ok = false; break; }
            tc_fence_after();
            const uint32_t sa = smem_u32(xs + kc * kAtChunk), sb = smem_u32(ws + s * kAtChunk);
#pragma unroll
            for (int kk = 0; kk < kBK / 16; kk++) {
              const uint64_t ah = smem_desc(sa + kk * 32), al = smem_desc(sa + kTileBytes + kk * 32);
              const uint64_t bh = smem_desc(sb + kk * 32), bl = smem_desc(sb + kTileBytes + kk * 32);
              mma_f16(d, ah, bh, (kc == 0 && kk == 0) ? 0u : 1u);
              mma_f16(d, ah, bl, 1u);
              mma_f16(d, al, bh, 1u);
            }
            mma_commit(&wempty[s]);
          }
        }
        if (!ok) break;
        mma_commit(xempty);
        mma_commit(accfull);
      }
      // every MMA this thread issued completes before TMEM is released
      mma_commit(drain);
      mbar_wait_drain(drain, 0);
    }
    __syncwarp();
  } else if (warp <= 3) {
    // ---------------- split: f32 boxes -> swizzled fp16 hi | lo, in place ----------------
    // Row r of the two [128 x 32] f32 boxes of a K-chunk occupies the same
    // bytes as row r of its hi and lo tiles, so a warp that reads a row
    // whole before writing it needs no other warp.
    const int sw = warp - 2;
    uint32_t tl = 0;
    bool ok = true;
    for (int k = blockIdx.x; k < a.tiles && ok; k += gridDim.x, tl++) {
      for (int kc = 0; kc < 2; kc++) {
        const bool mine = mbar_wait(&xraw[kc], tl & 1, a.err);
        if (!__all_sync(0xffffffffu, mine)) { ok = false; break; }
        unsigned char* base = xs + kc * kAtChunk;
        const int b = (lane >> 3) & 1, j = lane & 7;
        bool bad = false;
#pragma unroll 1
        for (int batch = 0; batch < 4; batch++) {
          float4 v[8];
#pragma unroll
          for (int p = 0; p < 8; p++) {
            const int r = sw * 64 + batch * 16 + p * 2 + (lane >> 4);
            v[p] = *reinterpret_cast<const float4*>(base + b * kTileBytes + r * 128 + ((j ^ (r & 7)) << 4));
          }
          __syncwarp();
#pragma unroll
          for (int p = 0; p < 8; p++) {
            const int r = sw * 64 + batch * 16 + p * 2 + (lane >> 4);
            float xv[4] = {v[p].x * a.a_scale, v[p].y * a.a_scale, v[p].z * a.a_scale, v[p].w * a.a_scale};
            float hi[4], lo[4];
#pragma unroll
            for (int e = 0; e < 4; e++) {
              bad |= !(fabsf(xv[e]) < 32768.0f);
              split_f32(xv[e], hi[e], lo[e]);
            }
            const uint32_t off = r * 128 + ((((4 * b + (j >> 1)) ^ (r & 7)) & 7) << 4) + (j & 1) * 8;
            *reinterpret_cast<uint2*>(base + off) =
                make_uint2(h2u(__floats2half2_rn(hi[0], hi[1])), h2u(__floats2half2_rn(hi[2], hi[3])));
            *reinterpret_cast<uint2*>(base + kTileBytes + off) =
                make_uint2(h2u(__floats2half2_rn(lo[0], lo[1])), h2u(__floats2half2_rn(lo[2], lo[3])));
          }
          __syncwarp();
        }
        if (bad) atomicOr(a.err, kErrOverflow);
        fence_proxy_async_smem();
        mbar_arrive(&xfull[kc]);
      }
    }
  } else {
    // ---------------- epilogue: attention + residual ----------------
    const int e = warp - 4, q = warp & 3, half = e >> 2;
    const int i = q * 32 + lane;  // this thread's row of the tile (its TMEM lane)
    const int bar_id = 2 + half;
    unsigned char* slot = kvs + half * kAtSlotBytes;
    unsigned char* rb = res + half * kAtResBytes;  // x[:, hd*32 .. +32] of the tile, TMA 128-byte swizzle
    const bool issuer = q == 0 && lane == 0;
    const uint32_t slot_u32 = smem_u32(slot);
    constexpr bool words = WORDS;
    const uint32_t lq = uint32_t(q * 32) << 16;
    uint32_t tl = 0;
    bool ok = true;
    // the next tile's rows and this thread's row info, loaded a tile ahead
    int nrow0 = 0, nrow1 = 0;
    uint32_t nrc = 0;
    if (int(blockIdx.x) < a.tiles) {
      nrow0 = a.tile_row[blockIdx.x];
      nrow1 = a.tile_row[blockIdx.x + 1];
      if (i < nrow1 - nrow0) nrc = a.row_rc[nrow0 + i];
    }
    for (int k = blockIdx.x; k < a.tiles && ok; k += gridDim.x, tl++) {
      const int row0 = nrow0;
      const int n = nrow1 - row0;
      const bool valid = i < n;
      const int s0 = i - int(nrc >> 4), cnt = int(nrc & 15u);
      if (k + int(gridDim.x) < a.tiles) {
        nrow0 = a.tile_row[k + gridDim.x];
        nrow1 = a.tile_row[k + gridDim.x + 1];
      }
      uint32_t wmine = KC_INVALID, wj[KC_RW];
#pragma unroll
      for (int j = 0; j < KC_RW; j++) wj[j] = KC_INVALID;
      if (valid && words) {
        const uint32_t tp = a.tok_recpos[row0 + i];
        wmine = a.word_ids[tp];
#pragma unroll
        for (int j = 0; j < KC_RW; j++)
          if (j < cnt) wj[j] = a.word_ids[a.tok_recpos[row0 + s0 + j]];
      }
      int okw = 0;
      if (lane == 0) okw = mbar_wait(accfull, tl & 1, a.err) ? 1 : 0;
      okw = __shfl_sync(0xffffffffu, okw, 0);
      int all;  // the half agrees before its named barriers
      asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %1, 0;\n\t"
                   "bar.red.and.pred p, %2, 128, p;\n\tselp.u32 %0, 1, 0, p;\n\t}"
                   : "=r"(all) : "r"(okw), "r"(bar_id) : "memory");
      if (!all) { ok = false; break; }
      tc_fence_after();
      if (k + int(gridDim.x) < a.tiles && i < nrow1 - nrow0) nrc = a.row_rc[nrow0 + i];
      const uint32_t qcol = (tl & 1) ? 384u : 0u;
#pragma unroll 1  // the two rounds as a loop: unrolled, the kernel spilled registers
      for (int r = 0; r < 2; r++) {
        const int hd = 2 * half + r;
        if (r == 1) named_bar(bar_id, 128);  // round 0 is done with the slot and the residual buffer
        if (issuer) {  // this round's residual columns, landing while the scores run
          mbar_arrive_expect_tx(&rfull[half], kAtResBytes);
          tma_load_2d(rb, &xmap, hd * 32, row0, &rfull[half]);
        }
        float4* mine_row = at_row(slot, i);
        {
          float t[32];
          tmem_ld32(tmem_base + lq + 128 + hd * 32, t);
#pragma unroll
          for (int m = 0; m < 8; m++)
            mine_row[m ^ (i & 15)] = make_float4(t[4 * m] * a.unscale, t[4 * m + 1] * a.unscale,
                                                 t[4 * m + 2] * a.unscale, t[4 * m + 3] * a.unscale);
          tmem_ld32(tmem_base + lq + 256 + hd * 32, t);
#pragma unroll
          for (int m = 0; m < 8; m++)
            mine_row[(8 + m) ^ (i & 15)] = make_float4(t[4 * m] * a.unscale, t[4 * m + 1] * a.unscale,
                                                       t[4 * m + 2] * a.unscale, t[4 * m + 3] * a.unscale);
        }
        if (r == 1) {
          tc_fence_before();
          mbar_arrive(kvempty);
        }
        float qv[32];
        tmem_ld32(tmem_base + lq + qcol + hd * 32, qv);
        if (r == 1) {
          tc_fence_before();
          mbar_arrive(&qempty[tl & 1]);
        }
        named_bar(bar_id, 128);  // the head's k | v rows are staged
        float4 o[8];
        if (valid) {
          float4 qq[8];
#pragma unroll
          for (int m = 0; m < 8; m++)
            qq[m] = make_float4(qv[4 * m] * a.unscale, qv[4 * m + 1] * a.unscale, qv[4 * m + 2] * a.unscale,
                                qv[4 * m + 3] * a.unscale);
          // all eight keys at once, so the eight 32-long fmaf chains interleave
          // (each keeps the order of the one-key-at-a-time loop); keys past the
          // record load nothing (zeros) and are masked out below
          uint32_t kr[KC_RW];
#pragma unroll
          for (int j = 0; j < KC_RW; j++) kr[j] = at_key(slot_u32, s0 + j);
          float p[KC_RW];
#pragma unroll
          for (int j = 0; j < KC_RW; j++) p[j] = 0.f;
#pragma unroll
          for (int m = 0; m < 8; m++)
#pragma unroll
            for (int j = 0; j < KC_RW; j++) {
              const float4 kv = lds4_if(kr[j] ^ (m << 4), j < cnt);
              p[j] = fmaf(qq[m].x, kv.x, p[j]); p[j] = fmaf(qq[m].y, kv.y, p[j]);
              p[j] = fmaf(qq[m].z, kv.z, p[j]); p[j] = fmaf(qq[m].w, kv.w, p[j]);
            }
          float mx = -INFINITY;
#pragma unroll
          for (int j = 0; j < KC_RW; j++) {
            p[j] = p[j] * a.scale;
            if (words) p[j] += word_bias(wmine, wj[j], a.word_alpha);
            if (j >= cnt) p[j] = -INFINITY;  // exp gives 0: adds nothing to the sum or the output
            mx = fmaxf(mx, p[j]);
          }
          float sum = 0.f;
#pragma unroll
          for (int j = 0; j < KC_RW; j++) { p[j] = expf(p[j] - mx); sum += p[j]; }
          // attentionOracle's all-blocked row (only a bias can block one): p = 0
          const float inv = words && !(mx >= -1e29f) ? 0.f : 1.f / fmaxf(sum, 1e-20f);
#pragma unroll
          for (int m = 0; m < 8; m++) o[m] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
          for (int j = 0; j < KC_RW; j++) {
            const float pj = p[j] * inv;
#pragma unroll
            for (int m = 0; m < 8; m++) {
              const float4 vv = lds4_if(kr[j] ^ ((8 + m) << 4), j < cnt);
              o[m].x = fmaf(pj, vv.x, o[m].x); o[m].y = fmaf(pj, vv.y, o[m].y);
              o[m].z = fmaf(pj, vv.z, o[m].z); o[m].w = fmaf(pj, vv.w, o[m].w);
            }
          }
        }
        // x += o on this thread's row, in the residual buffer
        mbar_wait(&rfull[half], uint32_t(r), a.err);
        if (valid) {
          float4* xr = reinterpret_cast<float4*>(rb + i * 128);
#pragma unroll
          for (int m = 0; m < 8; m++) {
            float4 xv = xr[m ^ (i & 7)];
            xv.x += o[m].x; xv.y += o[m].y; xv.z += o[m].z; xv.w += o[m].w;
            xr[m ^ (i & 7)] = xv;
          }
        }
        named_bar(bar_id, 128);  // the updated rows are in the buffer
        // coalesced stores: 8 lanes per row, 4 rows per instruction
        const int cl = lane & 7;
#pragma unroll
        for (int it = 0; it < 8; it++) {
          const int rr = q * 32 + (lane >> 3) + 4 * it;
          if (rr < n)
            *reinterpret_cast<float4*>(a.x + size_t(row0 + rr) * KC_H + hd * 32 + cl * 4) =
                reinterpret_cast<const float4*>(rb + rr * 128)[cl ^ (rr & 7)];
        }
      }
    }
    // a residual load left in flight by an expired wait lands before the CTA exits
    if (issuer && tl > 0) mbar_wait_drain(&rfull[half], 1u);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

// The x operand map of k_tc_attn: [rows x 128] f32, [128 rows x 32] boxes, 128-byte swizzle.
inline bool make_x_map(CUtensorMap* map, const float* x, uint64_t rows) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (!fn || (reinterpret_cast<uintptr_t>(x) & 15) || rows == 0) return false;
  const cuuint64_t dims[2] = {128, rows};
  const cuuint64_t strides[1] = {128 * 4};
  const cuuint32_t box[2] = {32, 128};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(x), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace tc
}  // namespace kc
