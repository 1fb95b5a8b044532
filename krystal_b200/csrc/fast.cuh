// fast.cuh — f32 SIMT kernels of the tensor-core path.
//
// The tensor-core path computes the forward to fp32-class accuracy (split
// fp16 GEMMs, f32 everywhere else) instead of the oracle's exact f64 order.
// Its distributions agree with the oracle to ~1e-6; its selections are
// CERTIFIED: k_select_fast bounds every score's distance from the exact
// computation's score by B_qj = kappa_q * scale * |sq_q| * |sk_j| + 4u|s_qj|
// and marks a question whose decision those bounds cannot settle (the top
// score's interval touching another's, a sampled draw within the cumulative
// error of a boundary, anything non-finite); the frames holding such
// questions are recomputed on the exact path. kappa_q = kappa0 * (1 +
// sqrt(Lambda_q / lam0)) grows with the question's largest |score| Lambda_q
// (sharper softmaxes upstream amplify relative errors).
#pragma once
#include "common.cuh"

namespace kc {

// ---------------------------------------------------------------------------
// Record-local attention + residual, f32 (attentionOracle local mode,
// forward/oracle.ts:64-105, :255-256). One warp per record. The record's
// q|k|v rows (contiguous, cnt x 1.5 KB) are staged in shared memory with
// coalesced 16-byte loads; float4 f of token row i is stored at f ^ i (an
// XOR swizzle within each aligned group of 8 float4), so the 8 lanes of a
// quarter-warp — one head, tokens 0..7 — read 8 different bank groups.
// lane = head*8 + token computes its scores, softmax and output in
// registers; the residual add then streams x with coalesced loads/stores.
// ---------------------------------------------------------------------------
constexpr int kLaWarps = 4;
constexpr int kLaRowF4 = 96;  // float4 per staged q|k|v row

struct LocalAttnFastArgs {
  const float* qkv;           // [T,384]
  float* x;                   // [T,128], updated in place
  const uint32_t* rec_start;  // [N]
  const uint2* rec_meta;      // [N]
  uint64_t records;
  float scale;                // 1/sqrt(headDim)
  const uint32_t* tok_recpos; // [T] record*8 | position, for the word ids
  const uint32_t* word_ids;   // optional [records*8]: the same-word bias's labels
  float word_alpha;
  float* p_out = nullptr;     // optional [T][4][8]: the softmax rows (saved for the backward)
};

__device__ __forceinline__ int la_swz(int row, int f4) { return row * kLaRowF4 + (f4 ^ row); }

__global__ void __launch_bounds__(kLaWarps * 32) k_local_attn_fast(LocalAttnFastArgs a) {
  __shared__ float4 stage[kLaWarps][KC_RW * kLaRowF4];  // 48 KB
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint64_t g = uint64_t(blockIdx.x) * kLaWarps + warp;
  if (g >= a.records) return;
  const uint32_t start = a.rec_start[g];
  const int cnt = int(a.rec_meta[g].y & 15u);
  if (cnt == 0) return;
  float4* st = stage[warp];
  // stage q|k|v with 16-byte asynchronous copies, every one of the record's in
  // flight at once; the residual rows load meanwhile
  const float4* src = reinterpret_cast<const float4*>(a.qkv + uint64_t(start) * 3 * KC_H);
  const int n4 = cnt * kLaRowF4;
  for (int i = lane; i < n4; i += 32) {
    const int r = i / kLaRowF4, f = i - r * kLaRowF4;
    const uint32_t dst = static_cast<uint32_t>(__cvta_generic_to_shared(st + la_swz(r, f)));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src + i) : "memory");
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  float4* xr = reinterpret_cast<float4*>(a.x + uint64_t(start) * KC_H);
  float4 xv[KC_RW];
#pragma unroll
  for (int r = 0; r < KC_RW; r++)
    if (r < cnt) xv[r] = xr[r * 32 + lane];
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncwarp();
  const int head = lane >> 3, ti = lane & 7;
  // word ids of the record's tokens: lane j (head 0) holds token j's
  uint32_t wmine = KC_INVALID, wj[KC_RW];
  const bool words = a.word_ids != nullptr;
  if (words) {
    if (ti < cnt) wmine = a.word_ids[a.tok_recpos[start + ti]];
#pragma unroll
    for (int j = 0; j < KC_RW; j++) wj[j] = __shfl_sync(0xffffffffu, wmine, j);
  }
  float4 o[8];
  if (ti < cnt) {
    float4 q[8];
#pragma unroll
    for (int m = 0; m < 8; m++) q[m] = st[la_swz(ti, head * 8 + m)];
    float p[KC_RW];
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < KC_RW; j++) {
      if (j < cnt) {
        float s = 0.f;
#pragma unroll
        for (int m = 0; m < 8; m++) {
          const float4 kv = st[la_swz(j, 32 + head * 8 + m)];
          s = fmaf(q[m].x, kv.x, s); s = fmaf(q[m].y, kv.y, s); s = fmaf(q[m].z, kv.z, s); s = fmaf(q[m].w, kv.w, s);
        }
        p[j] = s * a.scale;
        if (words) p[j] += word_bias(wmine, wj[j], a.word_alpha);
        mx = fmaxf(mx, p[j]);
      }
    }
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < KC_RW; j++)
      if (j < cnt) { p[j] = expf(p[j] - mx); sum += p[j]; }
    // attentionOracle's all-blocked row (only a bias can block one): p = 0
    const float inv = words && !(mx >= -1e29f) ? 0.f : 1.f / fmaxf(sum, 1e-20f);
#pragma unroll
    for (int m = 0; m < 8; m++) o[m] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int j = 0; j < KC_RW; j++) {
      if (j < cnt) {
        const float pj = p[j] * inv;
        if (a.p_out) a.p_out[((uint64_t(start) + ti) * KC_HEADS + head) * KC_RW + j] = pj;
#pragma unroll
        for (int m = 0; m < 8; m++) {
          const float4 vv = st[la_swz(j, 64 + head * 8 + m)];
          o[m].x = fmaf(pj, vv.x, o[m].x); o[m].y = fmaf(pj, vv.y, o[m].y);
          o[m].z = fmaf(pj, vv.z, o[m].z); o[m].w = fmaf(pj, vv.w, o[m].w);
        }
      }
    }
  }
  __syncwarp();
  if (ti < cnt) {  // only this lane read its q slice: it now holds the head's output
#pragma unroll
    for (int m = 0; m < 8; m++) st[la_swz(ti, head * 8 + m)] = o[m];
  }
  __syncwarp();
#pragma unroll
  for (int r = 0; r < KC_RW; r++)
    if (r < cnt) {
      const float4 ov = st[la_swz(r, lane)];
      xv[r].x += ov.x; xv[r].y += ov.y; xv[r].z += ov.z; xv[r].w += ov.w;
      xr[r * 32 + lane] = xv[r];
    }
}

// ---------------------------------------------------------------------------
// Learned-query pooling, f32 (poolRecord, oracle.ts:186-224). One warp per
// record; lane l holds dims 4l..4l+3 of each token row; the two score dot
// products are reduced across the warp.
// ---------------------------------------------------------------------------
struct PoolFastArgs {
  const float* x;
  const float* pool;          // [2,128]
  const uint32_t* rec_start;
  const uint2* rec_meta;
  const uint32_t* rec_row;    // bank row, or question row | 0x80000000
  uint64_t records;
  float scale;                // 1/sqrt(H)
  float* bank_keys;
  float* bank_values;
  float* query_values;
};

// The pooled key and value of one record from its rows xs[0..cnt) (lane l
// holding dims 4l..4l+3 of each row, zeros past cnt) and the two learned
// queries pk, pv (the lane's dims).
__device__ __forceinline__ void pool_record(const float4 (&xs)[KC_RW], int cnt, float4 pk, float4 pv, float scale,
                                            int lane, float4& ko_out, float4& vo_out) {
  float ks[KC_RW], vs[KC_RW];
#pragma unroll
  for (int j = 0; j < KC_RW; j++) {
    ks[j] = pk.x * xs[j].x + pk.y * xs[j].y + pk.z * xs[j].z + pk.w * xs[j].w;
    vs[j] = pv.x * xs[j].x + pv.y * xs[j].y + pv.z * xs[j].z + pv.w * xs[j].w;
  }
  // The sixteen lane partials (8 rows x the key and value queries), each
  // reduced over the 32 lanes by the xor butterfly 16, 8, 4, 2, 1 — transposed:
  // at each step a lane keeps half of its partial sums and hands the other
  // half to its partner, so the sixteen reductions take 16 shuffles instead
  // of 80 (and 16 to broadcast the totals). Every partial is formed from the
  // same two operands in the same order as in sixteen separate butterflies,
  // so the totals are bit-identical to them. Lane l ends with total l >> 1.
  {
    float v16[2 * KC_RW];
#pragma unroll
    for (int j = 0; j < KC_RW; j++) { v16[j] = ks[j]; v16[KC_RW + j] = vs[j]; }
    float a8[8], a4[4], a2[2];
    const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4, b1 = lane & 2;
#pragma unroll
    for (int i = 0; i < 8; i++) {
      const float keep = b4 ? v16[8 + i] : v16[i], send = b4 ? v16[i] : v16[8 + i];
      a8[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const float keep = b3 ? a8[4 + i] : a8[i], send = b3 ? a8[i] : a8[4 + i];
      a4[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
    }
#pragma unroll
    for (int i = 0; i < 2; i++) {
      const float keep = b2 ? a4[2 + i] : a4[i], send = b2 ? a4[i] : a4[2 + i];
      a2[i] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
    }
    const float keep = b1 ? a2[1] : a2[0], send = b1 ? a2[0] : a2[1];
    float t = keep + __shfl_xor_sync(0xffffffffu, send, 2);
    t += __shfl_xor_sync(0xffffffffu, t, 1);
#pragma unroll
    for (int j = 0; j < KC_RW; j++) {
      ks[j] = __shfl_sync(0xffffffffu, t, 2 * j);
      vs[j] = __shfl_sync(0xffffffffu, t, 2 * (KC_RW + j));
    }
  }
  float kmx = -INFINITY, vmx = -INFINITY;
#pragma unroll
  for (int j = 0; j < KC_RW; j++)
    if (j < cnt) {
      ks[j] *= scale;
      vs[j] *= scale;
      kmx = fmaxf(kmx, ks[j]);
      vmx = fmaxf(vmx, vs[j]);
    }
  float ksum = 0.f, vsum = 0.f;
#pragma unroll
  for (int j = 0; j < KC_RW; j++)
    if (j < cnt) {
      ks[j] = expf(ks[j] - kmx); ksum += ks[j];
      vs[j] = expf(vs[j] - vmx); vsum += vs[j];
    }
  const float kinv = cnt ? 1.f / fmaxf(ksum, 1e-20f) : 0.f, vinv = cnt ? 1.f / fmaxf(vsum, 1e-20f) : 0.f;
  float4 ko = make_float4(0.f, 0.f, 0.f, 0.f), vo = ko;
#pragma unroll
  for (int j = 0; j < KC_RW; j++)
    if (j < cnt) {
      const float kw = ks[j] * kinv, vw = vs[j] * vinv;
      ko.x = fmaf(kw, xs[j].x, ko.x); ko.y = fmaf(kw, xs[j].y, ko.y);
      ko.z = fmaf(kw, xs[j].z, ko.z); ko.w = fmaf(kw, xs[j].w, ko.w);
      vo.x = fmaf(vw, xs[j].x, vo.x); vo.y = fmaf(vw, xs[j].y, vo.y);
      vo.z = fmaf(vw, xs[j].z, vo.z); vo.w = fmaf(vw, xs[j].w, vo.w);
    }
  ko_out = ko;
  vo_out = vo;
}

__global__ void __launch_bounds__(256, 4) k_pool_fast(PoolFastArgs a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint64_t g = uint64_t(blockIdx.x) * 8 + warp;
  if (g >= a.records) return;
  const uint32_t start = a.rec_start[g];
  const int cnt = int(a.rec_meta[g].y & 15u);
  const uint32_t row = a.rec_row[g];
  const bool isq = row & 0x80000000u;
  const uint32_t r = row & 0x7fffffffu;
  float4* key_out = isq ? nullptr : reinterpret_cast<float4*>(a.bank_keys + uint64_t(r) * KC_H) + lane;
  float4* val_out = reinterpret_cast<float4*>(isq ? a.query_values + uint64_t(r) * KC_H
                                                  : a.bank_values + uint64_t(r) * KC_H) + lane;
  const float4 pk = __ldg(reinterpret_cast<const float4*>(a.pool) + lane);
  const float4 pv = __ldg(reinterpret_cast<const float4*>(a.pool + KC_H) + lane);
  // every row of the record in flight before any reduction
  float4 xs[KC_RW];
  const float4* xr = reinterpret_cast<const float4*>(a.x + uint64_t(start) * KC_H) + lane;
#pragma unroll
  for (int j = 0; j < KC_RW; j++) xs[j] = j < cnt ? __ldg(xr + j * 32) : make_float4(0.f, 0.f, 0.f, 0.f);
  float4 ko, vo;
  pool_record(xs, cnt, pk, pv, a.scale, lane, ko, vo);
  if (key_out) *key_out = ko;
  *val_out = vo;
}

// ---------------------------------------------------------------------------
// Mixer cross-attention + residual, f32 (oracle.ts:292-293 with the open
// mixer mask). One CTA per chunk of up to kCaChunk questions of a frame, the
// chunks of a frame adjacent in the grid so they share the bank in L2. The
// bank is streamed through shared memory in blocks of up to kCaBlock keys, so
// the chunk does not depend on the bank's length (a 4096-key bank is read by
// 4 CTAs per frame, not 64).
//
// Per (question, head): score j = the 32-long fmaf chain q·k_j in dimension
// order, scaled; softmax max and sum with lane l taking j = l, l+32, ... in
// key order, reduced by an xor-shuffle tree; output = (sum over even j of
// e_j v_j + sum over odd j of e_j v_j) / sum, each sum in key order, added to
// the question row. With more than one block, a first pass computes the
// scores for the row maxima only (a max does not depend on the order) and the
// second computes them again, identically, for the exponentials, the sums and
// p·v; every sum keeps its key order across the blocks (blocks start at
// multiples of 32 keys), so the result depends on neither the block size nor
// the thread tiling.
//
// Register tiles, so that each operand fetched from shared memory feeds
// several chains: a score thread holds 8 questions x 4 keys of one head (the
// warp: one head, 8 questions, 128 keys), a p·v thread 4 questions x 4
// columns of one key parity (the warp: 4 questions, all 128 columns).
//
// Shared memory: the k block, row j's float4 c at j*32 + (c ^ (j & 7)) (the
// score warp's lanes read 8 consecutive rows per quarter: 8 bank groups);
// the scores, row (question c, head) at (c*4 + head)*stride, key jj at
// (jj&1)*half + (jj>>1), so that a p·v chain reads four keys of its parity
// per float4 (half = 16 mod 32 keeps the score writes and the softmax reads
// free of bank conflicts); the chunk's question rows.
// ---------------------------------------------------------------------------
constexpr int kCaChunk = 16;
constexpr int kCaBlock = 128;
constexpr int kCaThreads = 256;
constexpr int kCaRowsPerWarp = kCaChunk * KC_HEADS / (kCaThreads / 32);

struct CrossAttnFrameArgs {
  const float* mq;
  const float* mk;
  const float* mv;
  float* query;
  const uint64_t* q_off;   // [frames + 1]
  const uint64_t* r_off;   // [frames + 1]
  int chunks;              // CTAs per frame: ceil(largest question count / kCaChunk)
  int kb;                  // keys per block: a multiple of 32, at most kCaBlock
  int half;                // the parity half's length in a score row (16 mod 32, >= kb/2)
  float scale;
};

__global__ void __launch_bounds__(kCaThreads, 2) k_cross_attn_frame(CrossAttnFrameArgs a) {
  extern __shared__ __align__(16) float4 caf_smem4[];  // k block [kCaBlock*32], scores, q [kCaChunk][32]
  __shared__ float inv_s[kCaChunk][KC_HEADS];
  const uint32_t f = blockIdx.x / a.chunks;
  const int q0 = int(blockIdx.x % a.chunks) * kCaChunk;
  const uint64_t qb = a.q_off[f], rb = a.r_off[f];
  const int nq = int(a.q_off[f + 1] - qb), R = int(a.r_off[f + 1] - rb);
  if (q0 >= nq) return;
  const int stride = 2 * a.half;
  float4* ks = caf_smem4;
  float* sc = reinterpret_cast<float*>(caf_smem4 + kCaBlock * 32);
  float* qs = sc + kCaChunk * KC_HEADS * stride;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nc = min(kCaChunk, nq - q0);
  const int nblk = (R + a.kb - 1) / a.kb;
  for (int i = tid; i < kCaChunk * KC_H; i += kCaThreads) qs[i] = i < nc * KC_H ? a.mq[(qb + q0) * KC_H + i] : 0.f;
  const float4* mk4 = reinterpret_cast<const float4*>(a.mk + rb * KC_H);
  auto stage = [&](int j0, int nb) {  // k rows [j0, j0 + nb) into the block buffer
    for (int i = tid; i < nb * 32; i += kCaThreads) {
      const int j = i >> 5, c4 = i & 31;
      cp_async16(ks + j * 32 + (c4 ^ (j & 7)), mk4 + size_t(j0 + j) * 32 + c4);
    }
  };
  auto staged = [&]() {
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();
  };

  // scores of the staged block: warp w takes head w/2 and questions
  // 8*(w&1) .. +7 (skipped when the chunk has none of them); lane l the keys
  // l, l+32, l+64, l+96 of the block
  const int s_head = warp >> 1, s_c0 = (warp & 1) * 8;
  auto scores = [&](int nb) {
    if (s_c0 >= nc) return;
    float acc[8][4];
#pragma unroll
    for (int c = 0; c < 8; c++)
#pragma unroll
      for (int t = 0; t < 4; t++) acc[c][t] = 0.f;
    const float4* q4p = reinterpret_cast<const float4*>(qs) + s_c0 * 32 + s_head * 8;
#pragma unroll 2
    for (int d4 = 0; d4 < KC_HEAD_DIM / 4; d4++) {
      float4 k4[4];
#pragma unroll
      for (int t = 0; t < 4; t++) {
        const int j = lane + 32 * t;
        k4[t] = ks[j * 32 + ((s_head * 8 + d4) ^ (j & 7))];
      }
#pragma unroll
      for (int c = 0; c < 8; c++) {
        const float4 q = q4p[c * 32 + d4];
#pragma unroll
        for (int t = 0; t < 4; t++) {
          acc[c][t] = fmaf(q.x, k4[t].x, acc[c][t]);
          acc[c][t] = fmaf(q.y, k4[t].y, acc[c][t]);
          acc[c][t] = fmaf(q.z, k4[t].z, acc[c][t]);
          acc[c][t] = fmaf(q.w, k4[t].w, acc[c][t]);
        }
      }
    }
#pragma unroll
    for (int t = 0; t < 4; t++) {
      const int jj = lane + 32 * t;
      if (jj < nb) {
        const int pos = (jj & 1) * a.half + (jj >> 1);
#pragma unroll
        for (int c = 0; c < 8; c++)
          if (s_c0 + c < nc) sc[((s_c0 + c) * KC_HEADS + s_head) * stride + pos] = acc[c][t] * a.scale;
      }
    }
  };
  auto at = [&](int rw, int jj) -> float& { return sc[rw * stride + (jj & 1) * a.half + (jj >> 1)]; };

  // rows (question, head) rw = warp + 8r belong to one warp for the whole kernel
  float mx[kCaRowsPerWarp], sum[kCaRowsPerWarp];
#pragma unroll
  for (int r = 0; r < kCaRowsPerWarp; r++) {
    mx[r] = -INFINITY;
    sum[r] = 0.f;
  }
  auto row_max = [&](int nb) {
#pragma unroll
    for (int r = 0; r < kCaRowsPerWarp; r++) {
      const int rw = warp + r * (kCaThreads / 32);
      if (rw < nc * KC_HEADS)
        for (int jj = lane; jj < nb; jj += 32) mx[r] = fmaxf(mx[r], at(rw, jj));
    }
  };
  auto reduce_max = [&]() {
#pragma unroll
    for (int r = 0; r < kCaRowsPerWarp; r++)
      for (int o = 16; o; o >>= 1) mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], o));
  };
  if (nblk > 1) {
    stage(0, min(a.kb, R));
    for (int b = 0; b < nblk; b++) {
      const int j0 = b * a.kb, nb = min(a.kb, R - j0);
      staged();
      scores(nb);
      __syncthreads();
      if (b + 1 < nblk) stage(j0 + a.kb, min(a.kb, R - j0 - a.kb));
      row_max(nb);
    }
    reduce_max();
  }

  // p·v: warp w takes questions 4*(w&3) .. +3 and key parity w>>2 (skipped
  // when the chunk has none of those questions); lane l columns 4l .. 4l+3
  const int v_c0 = (warp & 3) * 4, par = warp >> 2, col0 = lane * 4, v_head = lane >> 3;
  float acc[4][4];
#pragma unroll
  for (int c = 0; c < 4; c++)
#pragma unroll
    for (int i = 0; i < 4; i++) acc[c][i] = 0.f;
  if (nblk > 0) stage(0, min(a.kb, R));
  for (int b = 0; b < nblk; b++) {
    const int j0 = b * a.kb, nb = min(a.kb, R - j0);
    staged();
    scores(nb);
    __syncthreads();
    if (b + 1 < nblk) stage(j0 + a.kb, min(a.kb, R - j0 - a.kb));
    if (nblk == 1) {
      row_max(nb);
      reduce_max();
    }
#pragma unroll
    for (int r = 0; r < kCaRowsPerWarp; r++) {
      const int rw = warp + r * (kCaThreads / 32);
      if (rw < nc * KC_HEADS)
        for (int jj = lane; jj < nb; jj += 32) {
          float& s = at(rw, jj);
          const float e = expf(s - mx[r]);
          s = e;
          sum[r] += e;
        }
    }
    __syncthreads();
    if (v_c0 < nc) {
      const int npar = (nb - par + 1) >> 1;
      const float4* vp = reinterpret_cast<const float4*>(a.mv + (rb + j0 + par) * KC_H + col0);
      const float* srow = sc + v_head * stride + par * a.half;
      int e = 0;
      for (; e + 8 <= npar; e += 8) {  // 8 keys of this parity in flight per step
        float4 vv[8];
#pragma unroll
        for (int u = 0; u < 8; u++) vv[u] = vp[size_t(e + u) * (2 * KC_H / 4)];
#pragma unroll
        for (int c = 0; c < 4; c++) {
          const float4* s4 = reinterpret_cast<const float4*>(srow + (v_c0 + c) * KC_HEADS * stride + e);
          const float4 sa = s4[0], sb = s4[1];
          const float sv[8] = {sa.x, sa.y, sa.z, sa.w, sb.x, sb.y, sb.z, sb.w};
#pragma unroll
          for (int u = 0; u < 8; u++) {
            acc[c][0] = fmaf(sv[u], vv[u].x, acc[c][0]);
            acc[c][1] = fmaf(sv[u], vv[u].y, acc[c][1]);
            acc[c][2] = fmaf(sv[u], vv[u].z, acc[c][2]);
            acc[c][3] = fmaf(sv[u], vv[u].w, acc[c][3]);
          }
        }
      }
      for (; e < npar; e++) {
        const float4 v = vp[size_t(e) * (2 * KC_H / 4)];
#pragma unroll
        for (int c = 0; c < 4; c++) {
          const float s = srow[(v_c0 + c) * KC_HEADS * stride + e];
          acc[c][0] = fmaf(s, v.x, acc[c][0]);
          acc[c][1] = fmaf(s, v.y, acc[c][1]);
          acc[c][2] = fmaf(s, v.z, acc[c][2]);
          acc[c][3] = fmaf(s, v.w, acc[c][3]);
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < kCaRowsPerWarp; r++) {
    const int rw = warp + r * (kCaThreads / 32);
    for (int o = 16; o; o >>= 1) sum[r] += __shfl_xor_sync(0xffffffffu, sum[r], o);
    if (lane == 0 && rw < nc * KC_HEADS) inv_s[rw >> 2][rw & 3] = 1.f / fmaxf(sum[r], 1e-20f);
  }
  __syncthreads();  // the last block's p·v has read the scores; the q rows are free
  // the odd sums meet the even ones in the question buffer
  if (par == 1 && v_c0 < nc)
#pragma unroll
    for (int c = 0; c < 4; c++)
      reinterpret_cast<float4*>(qs)[(v_c0 + c) * 32 + lane] = make_float4(acc[c][0], acc[c][1], acc[c][2], acc[c][3]);
  __syncthreads();
  if (par == 0)
#pragma unroll
    for (int c = 0; c < 4; c++)
      if (v_c0 + c < nc) {
        const float4 o = reinterpret_cast<const float4*>(qs)[(v_c0 + c) * 32 + lane];
        const float is = inv_s[v_c0 + c][v_head];
        float4* dst = reinterpret_cast<float4*>(a.query + (qb + q0 + v_c0 + c) * KC_H) + lane;
        float4 y = *dst;
        y.x += (acc[c][0] + o.x) * is;
        y.y += (acc[c][1] + o.y) * is;
        y.z += (acc[c][2] + o.z) * is;
        y.w += (acc[c][3] + o.w) * is;
        *dst = y;
      }
}

// ---------------------------------------------------------------------------
// Mixer cross-attention for banks of at most kCsMaxBank keys: the same
// arithmetic as k_cross_attn_frame (bit for bit) in one pass, the chunk's
// scores for the whole bank held in shared memory, so that small frames need
// no second score pass. One CTA per chunk of up to kCsChunk questions (as
// many as the score buffer holds). The bank's k rows pass through shared
// memory in blocks of kCsKeys rows, copied asynchronously with coalesced
// 16-byte copies (row j's float4 c at c ^ (j & 7), so a warp reading one
// float4 of 32 rows meets 8 bank groups); a score thread takes one (key,
// head) of the block for every question of the chunk. p·v per output column,
// the even keys' sum on threads 0-127 and the odd keys' on 128-255, each in
// key order, every question of the chunk at once, v read straight from
// global memory (a warp reads 128 contiguous bytes of a row).
// ---------------------------------------------------------------------------
constexpr int kCsMaxBank = 256;
constexpr int kCsChunk = 8;
constexpr int kCsThreads = 256;
constexpr int kCsKeys = kCsThreads / KC_HEADS;  // keys per staged k block: one (key, head) per thread

struct CrossAttnSmallArgs {
  const float* mq;
  const float* mk;
  const float* mv;
  float* query;
  const uint64_t* q_off;   // [frames + 1]
  const uint64_t* r_off;   // [frames + 1]
  int qc;                  // questions per chunk
  int chunks;              // CTAs per frame: ceil(largest question count / qc)
  int half;                // a score row's parity half (16 mod 32, >= ceil(max_r / 2))
  float scale;
};

// Score rows here are parity-split like k_cross_attn_frame's: key j of row
// (c, head) at (c*4 + head)*2*half + (j&1)*half + (j>>1), so each p·v chain
// (one key parity) reads four keys per float4.
__global__ void __launch_bounds__(kCsThreads, 3) k_cross_attn_small(CrossAttnSmallArgs a) {
  extern __shared__ __align__(16) float cas_smem[];  // scores [qc][4][2*half], q [qc][128], k [kCsKeys][128]
  __shared__ float inv_s[kCsChunk][KC_HEADS];
  const uint32_t f = blockIdx.x / a.chunks;
  const int q0 = int(blockIdx.x % a.chunks) * a.qc;
  const uint64_t qb = a.q_off[f], rb = a.r_off[f];
  const int nq = int(a.q_off[f + 1] - qb), R = int(a.r_off[f + 1] - rb);
  if (q0 >= nq) return;
  const int stride = 2 * a.half;
  float* sc = cas_smem;
  float* qs = cas_smem + size_t(a.qc) * KC_HEADS * stride;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  auto at = [&](float* row, int j) -> float& { return row[(j & 1) * a.half + (j >> 1)]; };
  {
    const int nc = min(a.qc, nq - q0);
    for (int i = tid; i < nc * KC_H; i += kCsThreads) qs[i] = a.mq[(qb + q0) * KC_H + i];
    __syncthreads();
    // scores, a block of kCsKeys keys at a time: thread (head, key) of the
    // block, the 32-long fmaf chain in dimension order for every question of
    // the chunk (q from shared memory, a broadcast within the warp's head)
    {
    float4* kbuf = reinterpret_cast<float4*>(qs + size_t(a.qc) * KC_H);
    const int kh = tid / kCsKeys, jj = tid % kCsKeys, hb = kh * KC_HEAD_DIM;
    for (int kb0 = 0; kb0 < R; kb0 += kCsKeys) {
      const int nb = min(kCsKeys, R - kb0);
      for (int i = tid; i < nb * (KC_H / 4); i += kCsThreads) {
        const int j = i >> 5, c4 = i & 31;
        cp_async16(kbuf + j * 32 + (c4 ^ (j & 7)), a.mk + (rb + kb0 + j) * KC_H + c4 * 4);
      }
      asm volatile("cp.async.wait_all;" ::: "memory");
      __syncthreads();
      if (jj < nb) {
        float sa[kCsChunk];
#pragma unroll
        for (int c = 0; c < kCsChunk; c++) sa[c] = 0.f;
#pragma unroll 2
        for (int d4 = 0; d4 < KC_HEAD_DIM / 4; d4++) {
          const float4 x = kbuf[jj * 32 + ((kh * 8 + d4) ^ (jj & 7))];
#pragma unroll
          for (int c = 0; c < kCsChunk; c++)
            if (c < nc) {
              const float4 q4 = reinterpret_cast<const float4*>(qs + c * KC_H + hb)[d4];
              sa[c] = fmaf(q4.x, x.x, sa[c]);
              sa[c] = fmaf(q4.y, x.y, sa[c]);
              sa[c] = fmaf(q4.z, x.z, sa[c]);
              sa[c] = fmaf(q4.w, x.w, sa[c]);
            }
        }
#pragma unroll
        for (int c = 0; c < kCsChunk; c++)
          if (c < nc) at(sc + (c * KC_HEADS + kh) * stride, kb0 + jj) = sa[c] * a.scale;
      }
      __syncthreads();  // the block is read before the next one lands
    }
    }
    // softmax rows (question, head): one warp each
    for (int rw = warp; rw < nc * KC_HEADS; rw += kCsThreads / 32) {
      float* row = sc + size_t(rw) * stride;
      float mx = -INFINITY;
      for (int j = lane; j < R; j += 32) mx = fmaxf(mx, at(row, j));
      for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      float sum = 0.f;
      for (int j = lane; j < R; j += 32) {
        float& s = at(row, j);
        const float e = expf(s - mx);
        s = e;
        sum += e;
      }
      for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      if (lane == 0) inv_s[rw >> 2][rw & 3] = 1.f / fmaxf(sum, 1e-20f);
    }
    __syncthreads();
    // p·v per output column: threads 0-127 form the sum over the even keys and
    // threads 128-255 the sum over the odd keys (each in key order, every
    // question of the chunk at once, each v element loaded once for them);
    // the output adds the two, as the one-question-at-a-time form does
    {
      const int col = tid & (KC_H - 1), head = col >> 5, par = tid >> 7;
      float acc[kCsChunk];
#pragma unroll
      for (int c = 0; c < kCsChunk; c++) acc[c] = 0.f;
      const float* vcol = a.mv + (rb + par) * KC_H + col;
      const float* srow = sc + head * stride + par * a.half;
      const int npar = (R - par + 1) >> 1;  // keys of this parity
      int e = 0;
      for (; e + 16 <= npar; e += 16) {  // 16 keys of this parity in flight per step
        float vv[16];
#pragma unroll
        for (int u = 0; u < 16; u++) vv[u] = vcol[size_t(e + u) * (2 * KC_H)];
#pragma unroll
        for (int c = 0; c < kCsChunk; c++)
          if (c < nc) {
            const float4* s4 = reinterpret_cast<const float4*>(srow + c * KC_HEADS * stride + e);
#pragma unroll
            for (int u4 = 0; u4 < 4; u4++) {
              const float4 s = s4[u4];
              acc[c] = fmaf(s.x, vv[4 * u4 + 0], acc[c]);
              acc[c] = fmaf(s.y, vv[4 * u4 + 1], acc[c]);
              acc[c] = fmaf(s.z, vv[4 * u4 + 2], acc[c]);
              acc[c] = fmaf(s.w, vv[4 * u4 + 3], acc[c]);
            }
          }
      }
      for (; e < npar; e++) {
        const float va = vcol[size_t(e) * (2 * KC_H)];
#pragma unroll
        for (int c = 0; c < kCsChunk; c++)
          if (c < nc) acc[c] = fmaf(srow[c * KC_HEADS * stride + e], va, acc[c]);
      }
      // the odd sums meet the even ones in the (now free) question buffer
      if (par == 1)
#pragma unroll
        for (int c = 0; c < kCsChunk; c++)
          if (c < nc) qs[c * KC_H + col] = acc[c];
      __syncthreads();
      if (par == 0)
#pragma unroll
        for (int c = 0; c < kCsChunk; c++)
          if (c < nc) a.query[(qb + q0 + c) * KC_H + col] += (acc[c] + qs[c * KC_H + col]) * inv_s[c][head];
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// Pointer selector, f32, with certification (selectorOracle,
// forward/oracle.ts:332-382). One CTA of 256 threads per chunk of up to
// kSelChunk questions of a frame (the chunks of a frame adjacent in the grid,
// sharing the bank in L2): the chunk's scores are computed together so each
// bank key row is read once per chunk (per score: the 128-long fmaf chain in
// dimension order); then one warp per question: mask, top two, softmax (lane-
// strided sums reduced by an xor-shuffle tree), p, the argmax or the draw,
// and its certification. Writes p and the index, and raises flags[frame]
// when a decision is not certain.
// ---------------------------------------------------------------------------
constexpr int kSelChunk = 8;

struct SelectFastArgs {
  const float* sq;
  const float* sk;
  const uint64_t* r_off;
  const uint64_t* q_off;
  const uint64_t* p_off;
  const uint32_t* schema_allow;
  const uint32_t* band_allow;
  const uint32_t* bank_rec;
  const uint32_t* schema_ids;
  const uint32_t* band_ids;
  const float* mask;  // explicit mask laid out like p (exclusive with the rule), or null
  const double* uniforms;
  uint32_t max_r;
  int qc;           // questions per chunk (the score buffer holds qc x max_r)
  int chunks;       // CTAs per frame: ceil(largest question count / qc)
  float scale;
  const float* nq;  // [Q] |sq| of each question's projection (k_row_norms)
  const float* nk;  // [R] |sk| of each bank row's projection
  float kappa0;     // base relative error of the projections' dot product (see kCertKappa0)
  float lam0;       // score scale at which the amplification term reaches 1 (see kCertLam0)
  float* kappa;     // [Q] out: kappa_q, for the audit of recomputed frames
  float* p;
  uint32_t* index;
  uint32_t* flags;  // [frames]
  int scores_in_p;  // the raw dot products are already in p (k_select_scores_fast)
};

// The certification margin. Fast scores s^ differ from the exact path's s by
// first-order propagated rounding: the split-fp16 products (each within
// 3 * 2^-22 of the product, the dropped lo*lo term and the two splits) and the
// fp32 accumulations of the ~14 projection stages and the f32 attention /
// pooling / softmax stages on a question's path. Treating the rounding errors
// as independent and zero-mean (Higham & Mary, SIAM J. Sci. Comput. 41(5),
// 2019), a stage of inner dimension K contributes a relative row error of
// about (12 + sqrt(K/2)) u, u = 2^-24; fourteen such stages in quadrature
// give about 75 u = 4.5e-6 per row; at lambda = 5 standard deviations (a
// one-sided tail below 3e-7 per score) the rows sq, sk carry relative errors
// below 2.2e-5. |s^ - s| <= scale (|dsq||sk| + |sq||dsk|) (Cauchy-Schwarz,
// no credit for the random direction) then gives kappa0 = 2e-5 per score
// norm product, before the softmax term. Softmaxes with large logits L turn a
// relative logit error rho into an output change of order rho * L times the
// distribution's spread; the envelope 1 + sqrt(Lambda_q / lam0) (Lambda_q the
// question's largest |score|, which grows as the squared activation norm like
// every logit upstream) covers the measured growth of the error per norm
// product from 1x to 256x token rows with a margin of 3 or more. The margin
// is checked at run time: every recomputed frame is audited (k_cert_audit).
constexpr float kCertKappa0 = 2e-5f;
constexpr float kCertLam0 = 2.0f;
constexpr float kCertTie = 9.5367431640625e-07f;  // 2^-20: exact scores this far apart give distinct stored p

// |row| of each [rows, 128] f32 row, one warp per row, rounded up.
__global__ void __launch_bounds__(256) k_row_norms(const float* __restrict__ x, uint64_t rows,
                                                   float* __restrict__ out) {
  const uint64_t r = uint64_t(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (r >= rows) return;
  const int lane = threadIdx.x & 31;
  const float4 v = reinterpret_cast<const float4*>(x + r * KC_H)[lane];
  float s = v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  // an f32 sum of 128 squares is within 9 * 2^-24 of the true sum; 1 + 2^-19 covers it after the root
  if (lane == 0) out[r] = sqrtf(s) * 1.0000019073486328f;
}

// The selector's raw dot products q·k_j (the 128-long fmaf chain in dimension
// order, as k_select_fast forms them) for long banks: one CTA per chunk of up
// to kSsChunk questions of a frame, the chunks of a frame adjacent in the
// grid; the bank's key rows stream through shared memory in blocks of
// kSsBlock (float4 c of row j at j*32 + (c ^ (j & 7))), each loaded once for
// the chunk; warp w takes questions 8(w&1) .. +7 and keys 32(w>>1) + lane.
// The products go to the questions' p rows, where k_select_fast picks them up.
constexpr int kSsChunk = 16;
constexpr int kSsBlock = 128;
constexpr int kSsThreads = 256;
constexpr size_t kSsSmem = size_t(kSsBlock) * KC_H * 4 + size_t(kSsChunk) * KC_H * 4;

__global__ void __launch_bounds__(kSsThreads, 2) k_select_scores_fast(SelectFastArgs a, int chunks) {
  extern __shared__ __align__(16) float4 ss_smem[];
  float4* ks = ss_smem;
  const float4* qs4 = ss_smem + kSsBlock * 32;
  float* qs = reinterpret_cast<float*>(ss_smem + kSsBlock * 32);
  const uint32_t f = blockIdx.x / chunks;
  const int q0 = int(blockIdx.x % chunks) * kSsChunk;
  const uint64_t rb = a.r_off[f], qb = a.q_off[f];
  const int R = int(a.r_off[f + 1] - rb), nq = int(a.q_off[f + 1] - qb);
  if (q0 >= nq || R == 0) return;
  const int nc = min(kSsChunk, nq - q0);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int i = tid; i < kSsChunk * KC_H; i += kSsThreads) qs[i] = i < nc * KC_H ? a.sq[(qb + q0) * KC_H + i] : 0.f;
  const float4* sk4 = reinterpret_cast<const float4*>(a.sk + rb * KC_H);
  auto stage = [&](int j0) {
    const int nb = min(kSsBlock, R - j0);
    for (int i = tid; i < nb * 32; i += kSsThreads) {
      const int j = i >> 5, c4 = i & 31;
      cp_async16(ks + j * 32 + (c4 ^ (j & 7)), sk4 + size_t(j0 + j) * 32 + c4);
    }
  };
  const int c0 = (warp & 1) * 8, j = (warp >> 1) * 32 + lane;
  float* pbase = a.p + a.p_off[f] + uint64_t(q0) * R;
  const int nblk = (R + kSsBlock - 1) / kSsBlock;
  stage(0);
  for (int b = 0; b < nblk; b++) {
    const int j0 = b * kSsBlock, nb = min(kSsBlock, R - j0);
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();
    if (c0 < nc && j < nb) {
      float sv[8];
#pragma unroll
      for (int c = 0; c < 8; c++) sv[c] = 0.f;
#pragma unroll 2
      for (int d4 = 0; d4 < KC_H / 4; d4++) {
        const float4 k = ks[j * 32 + (d4 ^ (j & 7))];
#pragma unroll
        for (int c = 0; c < 8; c++) {
          const float4 q4 = qs4[(c0 + c) * 32 + d4];
          sv[c] = fmaf(q4.x, k.x, sv[c]);
          sv[c] = fmaf(q4.y, k.y, sv[c]);
          sv[c] = fmaf(q4.z, k.z, sv[c]);
          sv[c] = fmaf(q4.w, k.w, sv[c]);
        }
      }
#pragma unroll
      for (int c = 0; c < 8; c++)
        if (c0 + c < nc) pbase[uint64_t(c0 + c) * R + j0 + j] = sv[c];
    }
    __syncthreads();
    if (b + 1 < nblk) stage(j0 + kSsBlock);
  }
}

__global__ void __launch_bounds__(256) k_select_fast(SelectFastArgs a) {
  constexpr int NT = 256;
  extern __shared__ __align__(16) float sel_smem[];  // scores [qc][max_r], then q [qc][128]
  const uint32_t f = blockIdx.x / a.chunks;
  const int q0 = int(blockIdx.x % a.chunks) * a.qc;
  const uint64_t rb = a.r_off[f], qb = a.q_off[f];
  const int R = int(a.r_off[f + 1] - rb), nq = int(a.q_off[f + 1] - qb);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (q0 >= nq) return;
  if (R == 0) {
    for (int c = q0 + tid; c < min(nq, q0 + a.qc); c += NT) a.index[qb + c] = KC_INVALID;
    return;
  }
  float* qs = sel_smem + size_t(a.qc) * a.max_r;
  {
    const int nc = min(a.qc, nq - q0);
    if (a.scores_in_p) {  // k_select_scores_fast left the raw dot products in the p rows
      const float* src = a.p + a.p_off[f] + uint64_t(q0) * R;
      for (int c = 0; c < nc; c++)
        for (int j = tid; j < R; j += NT) sel_smem[size_t(c) * a.max_r + j] = src[uint64_t(c) * R + j];
    } else {
      for (int i = tid; i < nc * KC_H; i += NT) qs[i] = a.sq[(qb + q0) * KC_H + i];
    }
    __syncthreads();
    // raw dot products for the chunk: one key row per thread, read once
    for (int j = tid; j < R && !a.scores_in_p; j += NT) {
      const float4* kr = reinterpret_cast<const float4*>(a.sk + (rb + j) * KC_H);
      float sv[kSelChunk];
#pragma unroll
      for (int c = 0; c < kSelChunk; c++) sv[c] = 0.f;
#pragma unroll 4
      for (int d4 = 0; d4 < KC_H / 4; d4++) {
        const float4 k = kr[d4];
#pragma unroll
        for (int c = 0; c < kSelChunk; c++)
          if (c < nc) {
            const float4 q4 = reinterpret_cast<const float4*>(qs + c * KC_H)[d4];
            sv[c] = fmaf(q4.x, k.x, sv[c]);
            sv[c] = fmaf(q4.y, k.y, sv[c]);
            sv[c] = fmaf(q4.z, k.z, sv[c]);
            sv[c] = fmaf(q4.w, k.w, sv[c]);
          }
      }
#pragma unroll
      for (int c = 0; c < kSelChunk; c++)
        if (c < nc) sel_smem[size_t(c) * a.max_r + j] = sv[c];
    }
    __syncthreads();
    // one warp per question of the chunk: mask, top two, softmax, p, decision
    for (int c = warp; c < nc; c += NT / 32) {
      const uint64_t qi = qb + q0 + c;
      float* row = sel_smem + size_t(c) * a.max_r;
      float* prow = a.p + a.p_off[f] + uint64_t(q0 + c) * uint64_t(R);
      bool reopen = false;
      const uint32_t* sa = nullptr;
      uint32_t ba = 0;
      if (a.schema_allow) {
        sa = a.schema_allow + qi * 8;
        ba = a.band_allow[qi];
        uint32_t admitted = 0;
        for (int j = lane; j < R; j += 32) {
          const uint32_t gr = a.bank_rec[rb + j];
          const uint32_t s = a.schema_ids[gr], b = a.band_ids[gr];
          admitted += (s < 256u && b < 32u && ((sa[s >> 5] >> (s & 31)) & 1u) && ((ba >> b) & 1u)) ? 1u : 0u;
        }
        for (int o = 16; o; o >>= 1) admitted += __shfl_xor_sync(0xffffffffu, admitted, o);
        reopen = admitted == 0;
      }
      // scaled, masked scores; per-lane best (value, first index), the largest
      // |score| among admitted keys, and finiteness
      float b1 = -INFINITY, lam = 0.f;
      uint32_t i1 = KC_INVALID;
      int nonfinite = 0, open = 0;
      const float* mrow = a.mask ? a.mask + a.p_off[f] + uint64_t(q0 + c) * uint64_t(R) : nullptr;
      for (int j = lane; j < R; j += 32) {
        const float s = row[j];
        float m = 0.f;
        if (mrow) {
          m = mrow[j];
        } else if (sa && !reopen) {
          const uint32_t gr = a.bank_rec[rb + j];
          const uint32_t sid = a.schema_ids[gr], b = a.band_ids[gr];
          m = (sid < 256u && b < 32u && ((sa[sid >> 5] >> (sid & 31)) & 1u) && ((ba >> b) & 1u)) ? 0.f : -1e30f;
        }
        const float ss = s * a.scale;
        const float sc = ss + m;
        row[j] = sc;
        nonfinite |= !isfinite(s) || !isfinite(m);
        open |= sc >= -1e29f;
        if (m > -1e29f) lam = fmaxf(lam, fabsf(ss));
        if (sc > b1) { b1 = sc; i1 = uint32_t(j); }
      }
      // warp reduce: top value, index of the first top, Lambda_q, any-open, any-nonfinite
      for (int o = 16; o; o >>= 1) {
        const float ob1 = __shfl_xor_sync(0xffffffffu, b1, o);
        const uint32_t oi1 = __shfl_xor_sync(0xffffffffu, i1, o);
        if (ob1 > b1 || (ob1 == b1 && oi1 < i1)) { b1 = ob1; i1 = oi1; }
        lam = fmaxf(lam, __shfl_xor_sync(0xffffffffu, lam, o));
        nonfinite |= __shfl_xor_sync(0xffffffffu, nonfinite, o);
        open |= __shfl_xor_sync(0xffffffffu, open, o);
      }
      // the score bounds B_j: the top's own (bt), the largest s_j + B_j over the
      // other keys (hi), and the largest B_j (bmax, for draws)
      const float kap = a.kappa0 * (1.f + sqrtf(lam / a.lam0));
      const float qn = a.scale * a.nq[qi] * kap;
      float bt = 0.f, hi = -INFINITY, bmax = 0.f;
      for (int j = lane; j < R; j += 32) {
        const float sc = row[j];
        // + 4u|s|: the f32 roundings of the fast and the exact score, and of the
        // comparison below; an explicit mask adds the rounding of s*scale + m
        // (|s*scale| <= |s| + |m|)
        const float mag = mrow ? fabsf(sc) + fabsf(mrow[j]) : fabsf(sc);
        const float bj = qn * a.nk[rb + j] + 2.384185791015625e-07f * mag;
        if (sc >= -1e29f) bmax = fmaxf(bmax, bj);
        if (uint32_t(j) == i1) bt = bj;
        else hi = fmaxf(hi, sc + bj);
      }
      for (int o = 16; o; o >>= 1) {
        bt = fmaxf(bt, __shfl_xor_sync(0xffffffffu, bt, o));
        hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, o));
        bmax = fmaxf(bmax, __shfl_xor_sync(0xffffffffu, bmax, o));
      }
      // softmax (the all-blocked row keeps p = 0)
      float inv = 0.f;
      if (open) {
        float sum = 0.f;
        for (int j = lane; j < R; j += 32) {
          const float e = expf(row[j] - b1);
          row[j] = e;
          sum += e;
        }
        for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        inv = 1.f / fmaxf(sum, 1e-20f);
      }
      for (int j = lane; j < R; j += 32) {
        const float pv = open ? row[j] * inv : 0.f;
        row[j] = pv;
        prow[j] = pv;
      }
      __syncwarp();
      if (lane == 0) {
        bool certain = !nonfinite;
        uint32_t best;
        a.kappa[qi] = kap;
        if (!open) {
          best = KC_INVALID;  // every score below -1e29 on any accurate computation
        } else if (a.uniforms) {
          // sampleRow's inverse CDF; certain when the draw is clear of both edges
          // by more than the cumulative p can move: each p_j by at most
          // expm1(2 bmax) relative (its score and the normaliser's log); 8u for
          // the f32 roundings of e and p in both paths and expf's 2 ulp; the f32
          // rounding of expf's argument, sum_j p_j |s_j - s_max| u <= u log R
          // (at most 12u here, 16u allowed); the f32 normalising sum's
          // (R/32 + 5) u
          const float tau_c = expm1f(2.f * bmax) +
                              float((R + 31) / 32 + 5 + 24) * 5.9604644775390625e-08f;
          const double u = a.uniforms[qi];
          double cum = 0.0, prev = 0.0;
          int last = -1, drawn = -2;
          for (int j = 0; j < R; j++) {
            const double w = row[j];
            if (!(w > 0)) continue;
            last = j;
            prev = cum;
            cum += w;
            if (u < cum) { drawn = j; break; }
          }
          if (drawn == -2) {
            drawn = last;
            certain = certain && (u - cum > tau_c);
          } else {
            certain = certain && (cum - u > tau_c) && (u - prev > tau_c || drawn == 0);
          }
          // tiny weights near zero may flip between zero and positive
          best = drawn < 0 ? KC_INVALID : uint32_t(drawn);
        } else {
          // certain when the top score's interval clears every other's by the
          // tie margin: then the exact scores keep the order and the stored p too
          best = i1;
          certain = certain && (R == 1 || b1 - bt > hi + kCertTie);
        }
        a.index[qi] = best;
        if (!certain) atomicOr(&a.flags[f], 1u);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Audit of the certification margin on the frames recomputed exactly: for
// every (question, bank row) pair of listed frame list[blockIdx.x], the fast
// score (the selector's fmaf chain over the fast projections, scaled in f32)
// against the exact score (the f64 chain over the exact projections, rounded
// to f32), as a ratio to the margin B the selector allowed that pair
// (kappa_q * scale * |sq| * |sk| + 4u|s^|). The largest ratio goes to *out
// (non-negative float bits, so an unsigned max orders them). Unmasked: the
// audit measures score error, which the mask does not change.
//
// Tiled like a product: a CTA takes kAuChunk questions (blockIdx.z) x kAuKeys
// bank rows (blockIdx.y) of the frame, stages their fast and exact rows in
// shared memory with coalesced asynchronous copies (a key row's float4 c at
// c ^ (row & 7), so a warp reading one float4 of 32 rows meets 8 bank
// groups), and each thread forms 4 questions x 1 bank row, reading the key
// row once for the four.
// ---------------------------------------------------------------------------
constexpr int kAuChunk = 16;
constexpr int kAuKeys = 64;
constexpr int kAuSmem = 2 * (kAuChunk + kAuKeys) * KC_H * 4;  // fast and exact rows: 80 KB

__global__ void __launch_bounds__(256) k_cert_audit(
    const uint32_t* __restrict__ list, const uint64_t* __restrict__ q_off, const uint64_t* __restrict__ r_off,
    const uint64_t* __restrict__ sub_q_off, const uint64_t* __restrict__ sub_r_off, const float* __restrict__ fsq,
    const float* __restrict__ fsk, const float* __restrict__ esq, const float* __restrict__ esk,
    const float* __restrict__ nq, const float* __restrict__ nk, const float* __restrict__ kappa, float scale,
    double scale_d, unsigned* __restrict__ out) {
  extern __shared__ __align__(16) float au_smem[];
  __shared__ float red[8];
  const uint32_t f = list[blockIdx.x];
  const uint64_t qb = q_off[f], rb = r_off[f];
  const int Q = int(q_off[f + 1] - qb), R = int(r_off[f + 1] - rb);
  const int c0 = int(blockIdx.z) * kAuChunk, j0 = int(blockIdx.y) * kAuKeys;
  if (c0 >= Q || j0 >= R) return;
  const uint64_t eq = sub_q_off[blockIdx.x], er = sub_r_off[blockIdx.x];
  const int nc = min(kAuChunk, Q - c0), nj = min(kAuKeys, R - j0);
  float4* fq = reinterpret_cast<float4*>(au_smem);  // [kAuChunk][32]
  float4* xq = fq + kAuChunk * 32;                   // exact
  float4* fk = xq + kAuChunk * 32;                   // [kAuKeys][32], swizzled
  float4* xk = fk + kAuKeys * 32;                    // exact, swizzled
  const int tid = threadIdx.x;
  for (int i = tid; i < nc * 32; i += 256) {
    const int c = i >> 5, d4 = i & 31;
    cp_async16(fq + i, fsq + (qb + c0 + c) * KC_H + d4 * 4);
    cp_async16(xq + i, esq + (eq + c0 + c) * KC_H + d4 * 4);
  }
  for (int i = tid; i < nj * 32; i += 256) {
    const int j = i >> 5, d4 = i & 31, at = j * 32 + (d4 ^ (j & 7));
    cp_async16(fk + at, fsk + (rb + j0 + j) * KC_H + d4 * 4);
    cp_async16(xk + at, esk + (er + j0 + j) * KC_H + d4 * 4);
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncthreads();
  const int j = tid & (kAuKeys - 1), g = tid >> 6;  // bank row j; questions 4g .. 4g+3
  float worst = 0.f;
  if (j < nj && 4 * g < nc) {
    float sv[4] = {0.f, 0.f, 0.f, 0.f};
    double dv[4] = {0.0, 0.0, 0.0, 0.0};
    const float4* fkr = fk + j * 32;
    const float4* xkr = xk + j * 32;
    for (int d4 = 0; d4 < KC_H / 4; d4++) {
      const float4 b = fkr[d4 ^ (j & 7)], e = xkr[d4 ^ (j & 7)];
      const double ex = double(e.x), ey = double(e.y), ez = double(e.z), ew = double(e.w);
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const float4 a = fq[(4 * g + u) * 32 + d4], x = xq[(4 * g + u) * 32 + d4];
        sv[u] = fmaf(a.x, b.x, sv[u]);
        sv[u] = fmaf(a.y, b.y, sv[u]);
        sv[u] = fmaf(a.z, b.z, sv[u]);
        sv[u] = fmaf(a.w, b.w, sv[u]);
        dv[u] = fma(double(x.x), ex, dv[u]);
        dv[u] = fma(double(x.y), ey, dv[u]);
        dv[u] = fma(double(x.z), ez, dv[u]);
        dv[u] = fma(double(x.w), ew, dv[u]);
      }
    }
    const float nkj = nk[rb + j0 + j];
#pragma unroll
    for (int u = 0; u < 4; u++) {
      const int c = c0 + 4 * g + u;
      if (c >= Q) break;
      const float fs = sv[u] * scale;
      const float es = __double2float_rn(dv[u] * scale_d);
      const float bound = kappa[qb + c] * scale * nq[qb + c] * nkj + 2.384185791015625e-07f * fabsf(fs);
      const float r = fabsf(fs - es) / bound;
      if (r == r) worst = fmaxf(worst, r);  // a non-finite score was never certified
    }
  }
  for (int o = 16; o; o >>= 1) worst = fmaxf(worst, __shfl_xor_sync(0xffffffffu, worst, o));
  if ((tid & 31) == 0) red[tid >> 5] = worst;
  __syncthreads();
  if (tid == 0) {
    float m = 0.f;
    for (int w = 0; w < 8; w++) m = fmaxf(m, red[w]);
    atomicMax(out, __float_as_uint(m));
  }
}

// ---------------------------------------------------------------------------
// Fallback plumbing: gather the records of the frames to recompute into a
// compact batch, and scatter their exact results back.
// ---------------------------------------------------------------------------
// One CTA: sub_rec_off / sub_q_off / sub_p_off over the listed frames.
__global__ void k_fallback_offsets(const uint32_t* __restrict__ list, uint32_t n, const uint64_t* __restrict__ rec_off,
                                   const uint64_t* __restrict__ q_off, const uint64_t* __restrict__ p_off,
                                   uint64_t* __restrict__ sub_rec_off, uint64_t* __restrict__ sub_q_off,
                                   uint64_t* __restrict__ sub_p_off) {
  __shared__ unsigned long long tmp[32];
  unsigned long long br = 0, bq = 0, bp = 0;
  for (uint32_t c = 0; c < n; c += 1024) {
    const uint32_t i = c + threadIdx.x;
    unsigned long long r = 0, q = 0, pp = 0;
    if (i < n) {
      const uint32_t f = list[i];
      r = rec_off[f + 1] - rec_off[f];
      q = q_off[f + 1] - q_off[f];
      pp = p_off[f + 1] - p_off[f];
    }
    unsigned long long tr, tq, tp;
    const unsigned long long er = block_excl_scan<1024, unsigned long long>(r, &tr, tmp);
    const unsigned long long eq = block_excl_scan<1024, unsigned long long>(q, &tq, tmp);
    const unsigned long long ep = block_excl_scan<1024, unsigned long long>(pp, &tp, tmp);
    if (i < n) { sub_rec_off[i] = br + er; sub_q_off[i] = bq + eq; sub_p_off[i] = bp + ep; }
    br += tr; bq += tq; bp += tp;
  }
  if (threadIdx.x == 0) { sub_rec_off[n] = br; sub_q_off[n] = bq; sub_p_off[n] = bp; }
}

// One CTA per listed frame: its block of the explicit mask into the compact batch.
__global__ void k_fallback_mask(const uint32_t* __restrict__ list, const uint64_t* __restrict__ p_off,
                                const uint64_t* __restrict__ sub_p_off, const float* __restrict__ mask,
                                float* __restrict__ s_mask) {
  const uint32_t i = blockIdx.x, f = list[i];
  const uint64_t p0 = p_off[f], np = p_off[f + 1] - p0, d0 = sub_p_off[i];
  for (uint64_t k = threadIdx.x; k < np; k += blockDim.x) s_mask[d0 + k] = mask[p0 + k];
}

// One CTA per listed frame: copy its records (and its questions' rule rows
// and uniforms) into the compact batch.
__global__ void k_fallback_gather(const uint32_t* __restrict__ list, const uint64_t* __restrict__ rec_off,
                                  const uint64_t* __restrict__ q_off, const uint64_t* __restrict__ sub_rec_off,
                                  const uint64_t* __restrict__ sub_q_off, const uint32_t* __restrict__ token_ids,
                                  const uint32_t* __restrict__ field_roles, const uint32_t* __restrict__ schema_ids,
                                  const uint32_t* __restrict__ band_ids, const uint32_t* __restrict__ schema_allow,
                                  const uint32_t* __restrict__ band_allow, const double* __restrict__ uniforms,
                                  const uint32_t* __restrict__ word_ids,
                                  uint32_t* __restrict__ s_tok, uint32_t* __restrict__ s_role,
                                  uint32_t* __restrict__ s_schema, uint32_t* __restrict__ s_band,
                                  uint32_t* __restrict__ s_sallow, uint32_t* __restrict__ s_ballow,
                                  double* __restrict__ s_uni, uint32_t* __restrict__ s_words) {
  const uint32_t i = blockIdx.x, f = list[i];
  const uint64_t r0 = rec_off[f], n = rec_off[f + 1] - r0, d0 = sub_rec_off[i];
  for (uint64_t k = threadIdx.x; k < n * KC_RW; k += blockDim.x) {
    s_tok[d0 * KC_RW + k] = token_ids[r0 * KC_RW + k];
    s_role[d0 * KC_RW + k] = field_roles[r0 * KC_RW + k];
    if (word_ids) s_words[d0 * KC_RW + k] = word_ids[r0 * KC_RW + k];
  }
  for (uint64_t k = threadIdx.x; k < n; k += blockDim.x) {
    s_schema[d0 + k] = schema_ids[r0 + k];
    s_band[d0 + k] = band_ids[r0 + k];
  }
  const uint64_t q0 = q_off[f], nq = q_off[f + 1] - q0, e0 = sub_q_off[i];
  if (schema_allow) {
    for (uint64_t k = threadIdx.x; k < nq * 8; k += blockDim.x) s_sallow[e0 * 8 + k] = schema_allow[q0 * 8 + k];
    for (uint64_t k = threadIdx.x; k < nq; k += blockDim.x) s_ballow[e0 + k] = band_allow[q0 + k];
  }
  if (uniforms)
    for (uint64_t k = threadIdx.x; k < nq; k += blockDim.x) s_uni[e0 + k] = uniforms[q0 + k];
}

// Exact p blocks and indices back to the batch: a row of 32 CTAs per listed
// frame (blockIdx.x the frame, blockIdx.y its slice of the copy).
__global__ void k_fallback_scatter(const uint32_t* __restrict__ list, const uint64_t* __restrict__ p_off,
                                   const uint64_t* __restrict__ q_off, const uint64_t* __restrict__ sub_p_off,
                                   const uint64_t* __restrict__ sub_q_off, const float* __restrict__ sub_p,
                                   const uint32_t* __restrict__ sub_index, float* __restrict__ p,
                                   uint32_t* __restrict__ index) {
  const uint32_t i = blockIdx.x, f = list[i];
  const uint64_t np = p_off[f + 1] - p_off[f], nq = q_off[f + 1] - q_off[f];
  const uint64_t first = uint64_t(blockIdx.y) * blockDim.x + threadIdx.x, stride = uint64_t(gridDim.y) * blockDim.x;
  for (uint64_t k = first; k < np; k += stride) p[p_off[f] + k] = sub_p[sub_p_off[i] + k];
  for (uint64_t k = first; k < nq; k += stride) index[q_off[f] + k] = sub_index[sub_q_off[i] + k];
}

}  // namespace kc
