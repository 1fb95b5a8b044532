// backward.cuh — brainBackwardOracle (packages/krystal/src/forward/backward.ts:
// 751-982) as a session runs it (host/gradients.ts:30-66): context
// "available", the argument slot aimed at nothing (it contributes exactly
// zero), no route-kind labels, an open mixer mask.
//
// Same arithmetic contract as exact.cuh: one f64 accumulator per dot product
// walked in the reference's index order, f32 rounding wherever the reference
// stores into a Float32Array, and no contraction of a*b+c (the file is
// compiled with --fmad=false). fma() appears only where the product is of
// two f32 values, which is exact in f64, so fma equals multiply-then-add.
// Every kernel works on the packed batch layout of pack.cuh: compact tokens
// (t_off), questions (q_off), bank rows (r_off), and per-frame [Q_f, R_f]
// blocks at p_off.
//
// The backward's own dense products (gradients through Wq/Wk/Wv/W1/W2 and the
// selector projections) run on k_dgemm_exact with transposed weight copies;
// this file holds everything else.
#pragma once
#include "common.cuh"
#include "exact.cuh"

namespace kc {

// dst[k, n] = src[n, k]: the transposed copy a back-input product multiplies by
// (matmulBackInput, backward.ts:548-557, is dY · W = dY · (Wᵀ)ᵀ).
__global__ void __launch_bounds__(256) k_transpose(const float* __restrict__ src, float* __restrict__ dst, int n,
                                                  int k) {
  __shared__ float tile[32][33];
  const int k0 = blockIdx.x * 32, n0 = blockIdx.y * 32;
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int r = n0 + i, c = k0 + threadIdx.x;
    if (r < n && c < k) tile[i][threadIdx.x] = src[int64_t(r) * k + c];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int r = k0 + i, c = n0 + threadIdx.x;
    if (r < k && c < n) dst[int64_t(r) * n + c] = tile[threadIdx.x][i];
  }
}

// Shared batch geometry of the per-question / per-bank-row kernels.
struct BatchGeo {
  const uint32_t* query_frame;  // [Q]
  const uint32_t* bank_frame;   // [R]
  const uint64_t* q_off;        // [F+1]
  const uint64_t* r_off;        // [F+1]
  const uint64_t* p_off;        // [F+1]
};

// selectionMask (host/learn.ts:215-232) from the device rule: -1e30 where the
// rule forbids, 0 where it admits, and a row that admits nothing reopened to
// zeros (:229). One CTA per question.
struct RuleMaskArgs {
  BatchGeo g;
  const uint32_t* schema_allow;  // [Q*8]
  const uint32_t* band_allow;    // [Q]
  const uint32_t* bank_rec;      // bank row -> record
  const uint32_t* schema_ids;    // [records]
  const uint32_t* band_ids;      // [records]
  float* mask;                   // [P]
};

__global__ void __launch_bounds__(256) k_rule_mask(RuleMaskArgs a) {
  __shared__ uint32_t red[8];
  const uint32_t qi = blockIdx.x, f = a.g.query_frame[qi];
  const uint64_t rb = a.g.r_off[f];
  const int R = int(a.g.r_off[f + 1] - rb);
  float* row = a.mask + a.g.p_off[f] + (qi - a.g.q_off[f]) * uint64_t(R);
  const uint32_t* sa = a.schema_allow + uint64_t(qi) * 8;
  const uint32_t ba = a.band_allow[qi];
  auto admits = [&](int j) {
    const uint32_t rec = a.bank_rec[rb + j];
    const uint32_t s = a.schema_ids[rec], b = a.band_ids[rec];
    return s < 256u && b < 32u && ((sa[s >> 5] >> (s & 31)) & 1u) && ((ba >> b) & 1u);
  };
  uint32_t n = 0;
  for (int j = threadIdx.x; j < R; j += 256) n += admits(j) ? 1u : 0u;
  const bool reopen = block_sum_u32<256>(n, red) == 0;
  for (int j = threadIdx.x; j < R; j += 256) row[j] = reopen || admits(j) ? 0.0f : -1e30f;
}

// The critic's third input block, the mean bank value over what the selection
// allows (backward.ts:834-843, context "available"): a running f32 sum over
// the allowed rows in order, then one f64 division. Then the value head's
// prediction (decisionHeadOracle with one class, :845-852) over
// [queryOutput | gather | offered]. One CTA of 128 threads per question.
struct OfferedArgs {
  BatchGeo g;
  const float* mask;         // [P] the selection
  const float* bank_values;  // [R,128]
  const float* qout;         // [Q,128]
  const float* gather;       // [Q,128]
  const float* wv;           // value head [384]
  float* offered;            // [Q,128]
  uint32_t* n_allowed;       // [Q]
  float* pred;               // [Q]
};

__global__ void __launch_bounds__(128) k_offered_pred(OfferedArgs a) {
  __shared__ float ctx[3 * KC_H];
  const uint32_t qi = blockIdx.x, f = a.g.query_frame[qi];
  const uint64_t rb = a.g.r_off[f];
  const int R = int(a.g.r_off[f + 1] - rb);
  const float* mrow = a.mask + a.g.p_off[f] + (qi - a.g.q_off[f]) * uint64_t(R);
  const int d = threadIdx.x;
  float o = 0.0f;
  uint32_t n = 0;
  int j = 0;
  for (; j + 8 <= R; j += 8) {  // eight keys' loads in flight, the running sum in key order
    float mv[8], bv[8];
#pragma unroll
    for (int u = 0; u < 8; u++) {
      mv[u] = mrow[j + u];
      bv[u] = a.bank_values[(rb + j + u) * KC_H + d];
    }
#pragma unroll
    for (int u = 0; u < 8; u++)
      if (double(mv[u]) > -1e29) {
        o = f32(double(o) + double(bv[u]));
        n++;
      }
  }
  for (; j < R; j++) {
    if (double(mrow[j]) > -1e29) {
      o = f32(double(o) + double(a.bank_values[(rb + j) * KC_H + d]));
      n++;
    }
  }
  if (n) o = f32(double(o) / double(n));
  a.offered[uint64_t(qi) * KC_H + d] = o;
  if (d == 0) a.n_allowed[qi] = n;
  ctx[d] = a.qout[uint64_t(qi) * KC_H + d];
  ctx[KC_H + d] = a.gather[uint64_t(qi) * KC_H + d];
  ctx[2 * KC_H + d] = o;
  __syncthreads();
  if (d == 0) {
    double s = 0.0;
    for (int k = 0; k < 3 * KC_H; k++) s = fma(double(ctx[k]), double(a.wv[k]), s);
    a.pred[qi] = f32(s);
  }
}

// valueHeadLoss (backward.ts:49-62) per frame: the mean of 0.5·e² over the
// frame's questions and dPred = e / Q stored f32; no target (NaN valence) =
// no loss and no gradient.
__global__ void k_value_loss(const float* pred, const double* valence, const uint64_t* q_off, uint32_t frames,
                             float* dpred, double* loss) {
  const uint32_t f = blockIdx.x * blockDim.x + threadIdx.x;
  if (f >= frames) return;
  const uint64_t q0 = q_off[f];
  const uint32_t Q = uint32_t(q_off[f + 1] - q0);
  const double v = valence ? valence[f] : __longlong_as_double(0x7ff8000000000000ll);
  double l = 0.0;
  if (v == v && Q) {
    for (uint32_t i = 0; i < Q; i++) {
      const double e = double(pred[q0 + i]) - v;
      l += 0.5 * e * e;
      dpred[q0 + i] = f32(e / Q);
    }
    l /= Q;
  } else {
    for (uint32_t i = 0; i < Q; i++) dpred[q0 + i] = 0.0f;
  }
  loss[f] = l;
}

// dValueWv of decisionHeadBackward (backward.ts:459-506, C = 1): per frame,
// one f64 accumulator per input column over the frame's questions in order.
__global__ void __launch_bounds__(384) k_value_wv(const float* qout, const float* gather, const float* offered,
                                                 const float* dpred, const uint64_t* q_off, float* dwv) {
  const uint32_t f = blockIdx.x;
  const int dd = threadIdx.x;
  const uint64_t q0 = q_off[f], Q = q_off[f + 1] - q0;
  const float* src = dd < KC_H ? qout + dd : dd < 2 * KC_H ? gather + (dd - KC_H) : offered + (dd - 2 * KC_H);
  double s = 0.0;
  for (uint64_t i = 0; i < Q; i++) s = fma(double(dpred[q0 + i]), double(src[(q0 + i) * KC_H]), s);
  dwv[uint64_t(f) * 3 * KC_H + dd] = f32(s);
}

// decisionHeadBackward's input gradients (dQueryOut, dIntentGather,
// dAvailable = dPred·Wv blocks) and selectorBackwardScores (backward.ts:
// 293-336) for the intent slot: dP[j] = f32(dGather·V[j]); the row sum
// Σ p·(unrounded dot); dScore = f32(p·(dP − rowSum) + policy term), where the
// policy term is p − onehot for a target, sc·(onehot − p) with
// sc = pAway / max(1 − pAway, 1e-6) for an AWAY target (bit 31), 0 without.
// One CTA per question; dynamic shared memory 12 B × max_r (the dot products, then the p row).
struct SelBackArgs {
  BatchGeo g;
  const float* p;            // [P] policy
  const float* bank_values;  // [R,128]
  const float* wv;           // [384]
  const float* dpred;        // [Q]
  const uint32_t* targets;   // [Q] or null
  float* dquery;             // [Q,128] <- dQueryOut
  float* dig;                // [Q,128]
  float* dag;                // [Q,128]
  float* dscore;             // [P]
};

__global__ void __launch_bounds__(256) k_sel_back_scores(SelBackArgs a) {
  extern __shared__ __align__(16) unsigned char dyn[];
  double* s64 = reinterpret_cast<double*>(dyn);
  __shared__ double digs[KC_H];
  __shared__ double row_sum_s;
  const uint32_t qi = blockIdx.x, f = a.g.query_frame[qi];
  const uint64_t rb = a.g.r_off[f];
  const int R = int(a.g.r_off[f + 1] - rb);
  const uint64_t po = a.g.p_off[f] + (qi - a.g.q_off[f]) * uint64_t(R);
  const float* prow = a.p + po;
  const int tid = threadIdx.x;
  if (tid < KC_H) {
    const double dl = a.dpred[qi];
    const uint64_t o = uint64_t(qi) * KC_H + tid;
    const float vig = f32(dl * double(a.wv[KC_H + tid]));
    a.dquery[o] = f32(dl * double(a.wv[tid]));
    a.dig[o] = vig;
    a.dag[o] = f32(dl * double(a.wv[2 * KC_H + tid]));
    digs[tid] = vig;
  }
  float* ps = reinterpret_cast<float*>(s64 + R);  // the question's p row, staged once
  for (int j = tid; j < R; j += 256) ps[j] = prow[j];
  __syncthreads();
  for (int j = tid; j < R; j += 256) {
    const float* vr = a.bank_values + (rb + j) * KC_H;
    double s = 0.0;
#pragma unroll 8
    for (int d = 0; d < KC_H; d++) s = fma(digs[d], double(vr[d]), s);
    s64[j] = s;
  }
  __syncthreads();
  if (tid == 0) {
    double rs = 0.0;
    for (int j = 0; j < R; j++) rs = rs + double(ps[j]) * s64[j];
    row_sum_s = rs;
  }
  __syncthreads();
  const double row_sum = row_sum_s;
  const uint32_t raw = a.targets ? a.targets[qi] : KC_INVALID;
  const bool valid = raw != KC_INVALID;
  const bool away = valid && raw >= 0x80000000u;
  const uint32_t target = away ? raw - 0x80000000u : raw;
  const double p_away = away && target < uint32_t(R) ? double(ps[target]) : 0.0;
  const double sc = away ? p_away / js_max(1.0 - p_away, 1e-6) : 0.0;
  for (int j = tid; j < R; j += 256) {
    const double pij = ps[j];
    const double one = uint32_t(j) == target ? 1.0 : 0.0;
    const double pg = !valid ? 0.0 : away ? sc * (one - pij) : pij - one;
    a.dscore[po + j] = f32(pij * (double(f32(s64[j])) - row_sum) + pg);
  }
}

// selectorBackwardQkv (backward.ts:354-392), question side:
// dQProj[i,c] = f32(Σ_j dScore[i,j]·kProj[j,c] · 1/√H). One CTA per question.
__global__ void __launch_bounds__(128) k_sel_back_dq(BatchGeo g, const float* dscore, const float* sk, double hscale,
                                                    float* dqp) {
  const uint32_t qi = blockIdx.x, f = g.query_frame[qi];
  const uint64_t rb = g.r_off[f];
  const int R = int(g.r_off[f + 1] - rb);
  const float* drow = dscore + g.p_off[f] + (qi - g.q_off[f]) * uint64_t(R);
  const int c = threadIdx.x;
  double acc = 0.0;
  int j = 0;
  for (; j + 8 <= R; j += 8) {  // eight keys' loads in flight, the chain in key order
    float dv[8], kv[8];
#pragma unroll
    for (int u = 0; u < 8; u++) {
      dv[u] = drow[j + u];
      kv[u] = sk[(rb + j + u) * KC_H + c];
    }
#pragma unroll
    for (int u = 0; u < 8; u++) acc = fma(double(dv[u]), double(kv[u]), acc);
  }
  for (; j < R; j++) acc = fma(double(drow[j]), double(sk[(rb + j) * KC_H + c]), acc);
  dqp[uint64_t(qi) * KC_H + c] = f32(acc * hscale);
}

// selectorBackwardQkv, bank side, with the bank-value gradient assembled:
// dKProj[j,c] = f32(Σ_i dScore[i,j]·qProj[i,c] · 1/√H); the gather's
// dV2[j,c] = f32(Σ_i p[i,j]·dGather[i,c]); the offered mean's share
// dV1[j,c] = running f32 sum over questions allowing j of dAvailable/count;
// dBankValues = f32(dV1 + dV2) (backward.ts:890-898). One CTA per bank row.
struct SelBackKArgs {
  BatchGeo g;
  const float* dscore;      // [P]
  const float* p;           // [P]
  const float* mask;        // [P]
  const float* sq;          // [Q,128]
  const float* dig;         // [Q,128]
  const float* dag;         // [Q,128]
  const uint32_t* n_allowed;// [Q]
  double hscale;
  float* dkp;               // [R,128]
  float* dbv;               // [R,128]
  uint32_t rows;            // R: bank rows of the batch
};

constexpr int kSelBackRows = 8;  // bank rows per CTA of k_sel_back_dk

__global__ void __launch_bounds__(128) k_sel_back_dk(SelBackKArgs a) {
  const int c = threadIdx.x;
  // kSelBackRows bank rows per CTA (two in flight at a time); each row's
  // chains run over its frame's questions in order
#pragma unroll 2
  for (int r = 0; r < kSelBackRows; r++) {
    const uint32_t jg = blockIdx.x * kSelBackRows + r;
    if (jg >= a.rows) break;
    const uint32_t f = a.g.bank_frame[jg];
    const uint64_t rb = a.g.r_off[f];
    const uint64_t R = a.g.r_off[f + 1] - rb, j = jg - rb;
    const uint64_t q0 = a.g.q_off[f], Q = a.g.q_off[f + 1] - q0, pb = a.g.p_off[f];
    float dv1 = 0.0f;
    double ak = 0.0, av = 0.0;
    for (uint64_t i = 0; i < Q; i++) {
      const uint64_t pi = pb + i * R + j;
      const uint64_t qr = (q0 + i) * KC_H + c;
      if (double(a.mask[pi]) > -1e29) dv1 = f32(double(dv1) + double(a.dag[qr]) / double(a.n_allowed[q0 + i]));
      ak = fma(double(a.dscore[pi]), double(a.sq[qr]), ak);
      av = fma(double(a.p[pi]), double(a.dig[qr]), av);
    }
    a.dkp[uint64_t(jg) * KC_H + c] = f32(ak * a.hscale);
    a.dbv[uint64_t(jg) * KC_H + c] = f32(double(dv1) + double(f32(av)));
  }
}

// matmulBackWeight (backward.ts:560-569) per frame: dW_f[n,k] =
// f32(Σ_l dY[l,n]·X[l,k]) over the frame's rows l in order (row_off gives
// each frame's rows). Grid (frames, H/8); thread (k, 4 consecutive n).
__global__ void __launch_bounds__(256) k_weight_grad(const float* __restrict__ dY, const float* __restrict__ X,
                                                    const uint64_t* row_off, float* dW) {
  const uint32_t f = blockIdx.x;
  const int k = threadIdx.x & 127, n0 = blockIdx.y * 8 + (threadIdx.x >> 7) * 4;
  const uint64_t l0 = row_off[f], L = row_off[f + 1] - l0;
  double acc[4] = {0.0, 0.0, 0.0, 0.0};
  uint64_t l = 0;
  for (; l + 8 <= L; l += 8) {  // eight rows' loads in flight, each chain still in row order
    float x[8];
    float4 dy[8];
#pragma unroll
    for (int u = 0; u < 8; u++) {
      x[u] = X[(l0 + l + u) * KC_H + k];
      dy[u] = *reinterpret_cast<const float4*>(dY + (l0 + l + u) * KC_H + n0);
    }
#pragma unroll
    for (int u = 0; u < 8; u++) {
      acc[0] = fma(double(dy[u].x), double(x[u]), acc[0]);
      acc[1] = fma(double(dy[u].y), double(x[u]), acc[1]);
      acc[2] = fma(double(dy[u].z), double(x[u]), acc[2]);
      acc[3] = fma(double(dy[u].w), double(x[u]), acc[3]);
    }
  }
  for (; l < L; l++) {
    const double x = X[(l0 + l) * KC_H + k];
    const float* dy = dY + (l0 + l) * KC_H + n0;
#pragma unroll
    for (int m = 0; m < 4; m++) acc[m] = fma(double(dy[m]), x, acc[m]);
  }
  float* out = dW + uint64_t(f) * KC_H * KC_H;
#pragma unroll
  for (int m = 0; m < 4; m++) out[uint64_t(n0 + m) * KC_H + k] = f32(acc[m]);
}

// attentionBackwardScores + attentionBackwardQkv (backward.ts:79-166) for the
// mixer's dense cross-attention, question side. Per head: dP[j] =
// f32(dOut·V[j]), rowSum = Σ_j p·(unrounded dot), dS = f32(p·(dP − rowSum)),
// kept in ds [4][P]; dQ[i,c] = f32(Σ_j dS·K[j,c] · 1/√headDim).
// One CTA per question; dynamic shared memory 12 B × 4 × max_r.
struct CrossBackArgs {
  BatchGeo g;
  const float* dout;  // [Q,128]
  const float* mq;    // [Q,128]
  const float* mk;    // [R,128]
  const float* mv;    // [R,128]
  const float* p;     // [4][P]
  uint64_t total_p;
  uint32_t max_r;
  double scale;
  float* ds;          // [4][P]
  float* dq;          // [Q,128]
  float* dk;          // [R,128]
  float* dv;          // [R,128]
  uint32_t rows;      // R: bank rows of the batch (k_cross_attn_back_kv)
};

constexpr int kCrossBackRows = 8;  // bank rows per CTA of k_cross_attn_back_kv

__global__ void __launch_bounds__(128) k_cross_attn_back_q(CrossBackArgs a) {
  extern __shared__ __align__(16) unsigned char dyn[];
  double* s64 = reinterpret_cast<double*>(dyn);                     // [4][max_r]
  float* dss = reinterpret_cast<float*>(s64 + 4 * size_t(a.max_r));  // [4][max_r]: the question's p rows, then dS
  __shared__ float dos[KC_H];
  __shared__ double rsum[KC_HEADS];
  const uint32_t qi = blockIdx.x, f = a.g.query_frame[qi];
  const uint64_t rb = a.g.r_off[f];
  const int R = int(a.g.r_off[f + 1] - rb);
  const uint64_t po = a.g.p_off[f] + (qi - a.g.q_off[f]) * uint64_t(R);
  const int tid = threadIdx.x;
  dos[tid] = a.dout[uint64_t(qi) * KC_H + tid];
  for (int idx = tid; idx < R * KC_HEADS; idx += 128) {  // p rows staged once (coalesced per head)
    const int head = idx / R, j = idx - head * R;
    dss[head * size_t(a.max_r) + j] = a.p[uint64_t(head) * a.total_p + po + j];
  }
  __syncthreads();
  for (int idx = tid; idx < R * KC_HEADS; idx += 128) {
    const int j = idx >> 2, head = idx & 3, hb = head * KC_HEAD_DIM;
    const float* vr = a.mv + (rb + j) * KC_H + hb;
    double s = 0.0;
#pragma unroll 8
    for (int d = 0; d < KC_HEAD_DIM; d++) s = fma(double(dos[hb + d]), double(vr[d]), s);
    s64[head * size_t(a.max_r) + j] = s;
  }
  __syncthreads();
  if (tid < KC_HEADS) {
    const float* prow = dss + tid * size_t(a.max_r);
    const double* sr = s64 + tid * size_t(a.max_r);
    double rs = 0.0;
    for (int j = 0; j < R; j++) rs = rs + double(prow[j]) * sr[j];
    rsum[tid] = rs;
  }
  __syncthreads();
  for (int idx = tid; idx < R * KC_HEADS; idx += 128) {
    const int head = idx / R, j = idx - head * R;
    const uint64_t pi = uint64_t(head) * a.total_p + po + j;
    float* slot = dss + head * size_t(a.max_r) + j;
    const double pij = *slot;
    const float v = f32(pij * (double(f32(s64[head * size_t(a.max_r) + j])) - rsum[head]));
    *slot = v;
    a.ds[pi] = v;
  }
  __syncthreads();
  const int head = tid >> 5;
  const float* dr = dss + head * size_t(a.max_r);
  const float* mkc = a.mk + rb * KC_H + tid;
  double acc = 0.0;
  int j = 0;
  for (; j + 16 <= R; j += 16) {  // sixteen keys' loads in flight, the chain in key order
    float kv[16];
#pragma unroll
    for (int u = 0; u < 16; u++) kv[u] = mkc[size_t(j + u) * KC_H];
#pragma unroll
    for (int u = 0; u < 16; u++) acc = fma(double(dr[j + u]), double(kv[u]), acc);
  }
  for (; j < R; j++) acc = fma(double(dr[j]), double(mkc[size_t(j) * KC_H]), acc);
  a.dq[uint64_t(qi) * KC_H + tid] = f32(acc * a.scale);
}

// The key/value side: dK[j,c] = f32(Σ_i dS·Q[i,c] · 1/√headDim),
// dV[j,c] = f32(Σ_i p·dOut[i,c]), i over the frame's questions in order.
// One CTA per bank row; warp w is head w.
__global__ void __launch_bounds__(128) k_cross_attn_back_kv(CrossBackArgs a) {
  const int col = threadIdx.x, head = col >> 5;
  // kCrossBackRows bank rows per CTA (two in flight at a time); each row's
  // chains run over its frame's questions in order
#pragma unroll 2
  for (int r = 0; r < kCrossBackRows; r++) {
    const uint32_t jg = blockIdx.x * kCrossBackRows + r;
    if (jg >= a.rows) break;
    const uint32_t f = a.g.bank_frame[jg];
    const uint64_t rb = a.g.r_off[f];
    const uint64_t R = a.g.r_off[f + 1] - rb, j = jg - rb;
    const uint64_t q0 = a.g.q_off[f], Q = a.g.q_off[f + 1] - q0;
    const uint64_t base = uint64_t(head) * a.total_p + a.g.p_off[f] + j;
    double ak = 0.0, av = 0.0;
    for (uint64_t i = 0; i < Q; i++) {
      const uint64_t pi = base + i * R;
      const uint64_t qr = (q0 + i) * KC_H + col;
      ak = fma(double(a.ds[pi]), double(a.mq[qr]), ak);
      av = fma(double(a.p[pi]), double(a.dout[qr]), av);
    }
    a.dk[uint64_t(jg) * KC_H + col] = f32(ak * a.scale);
    a.dv[uint64_t(jg) * KC_H + col] = f32(av);
  }
}

// poolBackward (backward.ts:184-262) for every record: the two pooling
// softmaxes are recomputed as the forward computed them; dP = f32(dOut·s_j),
// dS = p·(dP − Σ p·dP), the token-state gradient
// f32(pk·dKey + pv·dValue + 1/√H·(dSk·pool_k + dSv·pool_v)), and dSk/dSv kept
// per token for the pool-weight gradient. Bank records take the bank-key and
// bank-value gradients; questions take a zero key gradient and the query
// gradient (backward.ts:944-950). One warp per record.
struct PoolBackArgs {
  const float* x;            // [T,128] the encoder's output
  const float* pool;         // [2,128]
  const uint32_t* rec_start;
  const uint2* rec_meta;
  const uint32_t* rec_row;   // bank row, or question row | 0x80000000
  uint64_t records;
  double scale;              // 1/sqrt(H)
  const float* dbk;          // [R,128]
  const float* dbv;          // [R,128]
  const float* dquery;       // [Q,128]
  float* dfs;                // [T,128]
  double* tok_ds;            // [T][2]
};

__global__ void __launch_bounds__(256) k_pool_back(PoolBackArgs a) {
  __shared__ float xs[8][KC_RW][KC_H];  // 32 KB
  __shared__ float ps[2][KC_H];
  __shared__ float pr[8][2][KC_RW];     // pooling softmax rows (pk, pv)
  __shared__ float dp[8][2][KC_RW];     // dPk, dPv
  __shared__ double dsm[8][2][KC_RW];   // dSk, dSv
  __shared__ double rsm[8][2];
  __shared__ float gs[8][2][KC_H];      // the record's dKey (0 for a question) and dValue rows
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < 2 * KC_H; i += 256) (&ps[0][0])[i] = a.pool[i];
  __syncthreads();
  const uint64_t g = uint64_t(blockIdx.x) * 8 + warp;
  if (g >= a.records) return;
  const uint32_t start = a.rec_start[g];
  const int cnt = int(a.rec_meta[g].y & 15u);
  if (cnt == 0) return;
  const uint32_t row = a.rec_row[g];
  const bool isq = row & 0x80000000u;
  const uint32_t r = row & 0x7fffffffu;
  const float* dkey = isq ? nullptr : a.dbk + uint64_t(r) * KC_H;
  const float* dval = isq ? a.dquery + uint64_t(r) * KC_H : a.dbv + uint64_t(r) * KC_H;
  const float4* src = reinterpret_cast<const float4*>(a.x + uint64_t(start) * KC_H);
  float4* dst = reinterpret_cast<float4*>(&xs[warp][0][0]);
  for (int i = lane; i < cnt * 32; i += 32) dst[i] = src[i];
  for (int d = lane; d < KC_H; d += 32) {
    gs[warp][0][d] = dkey ? dkey[d] : 0.0f;
    gs[warp][1][d] = dval[d];
  }
  __syncwarp();
  const int j = lane & 7, which = lane >> 3;  // lanes 0..15 work
  if (lane < 16 && j < cnt) {
    double s = 0.0;
    for (int d = 0; d < KC_H; d++) s = fma(double(ps[which][d]), double(xs[warp][j][d]), s);
    pr[warp][which][j] = f32(s * a.scale);
  }
  __syncwarp();
  if (lane == 0 || lane == 8) softmax_small(pr[warp][lane >> 3], cnt);
  __syncwarp();
  if (lane < 16 && j < cnt) {
    const float* gr = gs[warp][which];
    double s = 0.0;
    for (int d = 0; d < KC_H; d++) s = fma(double(gr[d]), double(xs[warp][j][d]), s);
    dp[warp][which][j] = f32(s);
  }
  __syncwarp();
  if (lane == 0 || lane == 8) {
    const int w = lane >> 3;
    double rs = 0.0;
    for (int i = 0; i < cnt; i++) rs = fma(double(pr[warp][w][i]), double(dp[warp][w][i]), rs);
    rsm[warp][w] = rs;
  }
  __syncwarp();
  if (lane < 16 && j < cnt) {
    const double v = double(pr[warp][which][j]) * (double(dp[warp][which][j]) - rsm[warp][which]);
    dsm[warp][which][j] = v;
    a.tok_ds[(uint64_t(start) + j) * 2 + which] = v;
  }
  __syncwarp();
  for (int d = lane; d < KC_H; d += 32) {
    const double gk = double(gs[warp][0][d]), gv = double(gs[warp][1][d]);
    const double pk_d = ps[0][d], pv_d = ps[1][d];
    for (int t = 0; t < cnt; t++) {
      const double ds = double(pr[warp][0][t]) * gk + double(pr[warp][1][t]) * gv +
                        a.scale * (dsm[warp][0][t] * pk_d + dsm[warp][1][t] * pv_d);
      a.dfs[(uint64_t(start) + t) * KC_H + d] = f32(0.0 + ds);
    }
  }
}

// The pool-weight gradient per frame: for column c of [2,H], a running f32
// sum of 1/√H·dS·s over the frame's bank records, then (separately) its
// questions, each in order, token by token; dPool = f32(f32(0 + bank) +
// questions) (backward.ts:944-953). One CTA of 256 threads per frame.
struct PoolGradArgs {
  const float* x;
  const double* tok_ds;
  const uint32_t* rec_start;
  const uint2* rec_meta;
  const uint32_t* bank_rec;
  const uint32_t* query_rec;
  const uint64_t* r_off;
  const uint64_t* q_off;
  double scale;
  float* dpool;  // [F, 2H]
};

constexpr int kPoolGradChunk = 1024;  // records whose start and count are staged at a time

__global__ void __launch_bounds__(256) k_pool_grad(PoolGradArgs a) {
  __shared__ uint2 meta[kPoolGradChunk];  // (first token, token count) of the chunk's records
  const uint32_t f = blockIdx.x;
  const int c = threadIdx.x, which = c >> 7, d = c & 127;
  // the running f32 sum over the list's records and their tokens, in order;
  // the record list is staged a chunk at a time, and each record's terms are
  // loaded together, the next record's while this one is summed
  auto walk = [&](const uint32_t* list, uint64_t b, uint64_t e) {
    float acc = 0.0f;
    for (uint64_t c0 = b; c0 < e; c0 += kPoolGradChunk) {
      const int n = int(e - c0 < uint64_t(kPoolGradChunk) ? e - c0 : uint64_t(kPoolGradChunk));
      __syncthreads();  // the previous chunk's walk is done with meta
      for (int i = c; i < n; i += 256) {
        const uint32_t g = list[c0 + i];
        meta[i] = make_uint2(a.rec_start[g], a.rec_meta[g].y & 15u);
      }
      __syncthreads();
      float xn[KC_RW];
      double dn[KC_RW];
      auto fetch = [&](int r) {
        const uint2 m = meta[r];
#pragma unroll
        for (int t = 0; t < KC_RW; t++)
          if (t < int(m.y)) {
            const uint64_t tok = uint64_t(m.x) + t;
            xn[t] = a.x[tok * KC_H + d];
            dn[t] = a.tok_ds[tok * 2 + which];
          }
      };
      fetch(0);
      for (int r = 0; r < n; r++) {
        float xc[KC_RW];
        double dc[KC_RW];
#pragma unroll
        for (int t = 0; t < KC_RW; t++) {
          xc[t] = xn[t];
          dc[t] = dn[t];
        }
        const int cnt = int(meta[r].y);
        if (r + 1 < n) fetch(r + 1);
#pragma unroll
        for (int t = 0; t < KC_RW; t++) {
          if (t >= cnt) break;
          acc = f32(double(acc) + a.scale * dc[t] * double(xc[t]));
        }
      }
    }
    return acc;
  };
  const float b = walk(a.bank_rec, a.r_off[f], a.r_off[f + 1]);
  const float q = walk(a.query_rec, a.q_off[f], a.q_off[f + 1]);
  a.dpool[uint64_t(f) * 2 * KC_H + c] = f32(double(f32(0.0 + double(b))) + double(q));
}

// attentionBackwardScores + attentionBackwardQkv for the encoder's record-
// local attention (backward.ts:79-166, local windows): per record, head and
// token, dS over the record's keys from the saved p; then dQ, dK, dV of every
// token of the record, each one accumulator over the record in order.
// One warp per record; outputs dq | dk | dv as [T,384].
struct LocalBackArgs {
  const float* qkv;          // saved [T,384]
  const float* p;            // saved [T][4][8]
  const float* dout;         // [T,128]
  const uint32_t* rec_start;
  const uint2* rec_meta;
  uint64_t records;
  double scale;              // 1/sqrt(headDim)
  float* dqkv;               // [T,384]
};

constexpr int kLocalBackWarps = 4;
// per warp: p and dS of one record, then its q|k|v rows (8 x 96 float4) and
// dOut rows (8 x 32 float4)
constexpr int kLocalBackWarpFloats = 2 * KC_HEADS * KC_RW * KC_RW + KC_RW * (96 + 32) * 4;
constexpr size_t kLocalBackSmem = size_t(kLocalBackWarps) * kLocalBackWarpFloats * 4;

// Staged dOut row r of a record: 32 float4 (heads 0-3, 8 float4 each), float4
// m of head h at h*8 + ((m + 2h + (r & 1)) & 7) — the dOut analogue of
// la_exact_f4, so a quarter-warp (two tokens x four heads) reads 8 bank groups.
__device__ __forceinline__ int lb_dout_f4(int r, int f) {
  return r * 32 + (f & ~7) + (((f & 7) + 2 * ((f >> 3) & 3) + (r & 1)) & 7);
}

// One warp per record, 4 warps per CTA. The record's q|k|v and dOut rows
// (at most 16 KB) are staged in shared memory with one batch of asynchronous
// 16-byte copies, so each record costs one round trip to memory; the scores,
// dS and the dQ | dK | dV chains then read shared memory only. A = double is
// the oracle's arithmetic (the exact backward); A = float the same chains in
// f32, for the tensor-core backward, whose products are fp32-class already.
template <typename A>
__global__ void __launch_bounds__(kLocalBackWarps * 32, 3) k_local_attn_back(LocalBackArgs a) {
  extern __shared__ __align__(16) float lsm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint64_t g = uint64_t(blockIdx.x) * kLocalBackWarps + warp;
  if (g >= a.records) return;
  const uint32_t start = a.rec_start[g];
  const int cnt = int(a.rec_meta[g].y & 15u);
  if (cnt == 0) return;
  float* wsm = lsm + size_t(warp) * kLocalBackWarpFloats;
  float(*pp)[KC_RW][KC_RW] = reinterpret_cast<float(*)[KC_RW][KC_RW]>(wsm);
  float(*dsh)[KC_RW][KC_RW] = pp + KC_HEADS;  // [head][i][j]
  float4* rows = reinterpret_cast<float4*>(wsm + 2 * KC_HEADS * KC_RW * KC_RW);  // q|k|v, la_exact_f4 layout
  float4* drows = rows + KC_RW * 96;                                              // dOut, lb_dout_f4 layout
  {
    const float4* src = reinterpret_cast<const float4*>(a.qkv + uint64_t(start) * 3 * KC_H);
    for (int i = lane; i < cnt * 96; i += 32) cp_async16(rows + la_exact_f4(i / 96, i % 96), src + i);
    const float4* dsrc = reinterpret_cast<const float4*>(a.dout + uint64_t(start) * KC_H);
    for (int i = lane; i < cnt * 32; i += 32) cp_async16(drows + lb_dout_f4(i >> 5, i & 31), dsrc + i);
  }
  for (int i = lane; i < cnt * KC_HEADS * KC_RW; i += 32) {
    const int ti = i >> 5, head = (i >> 3) & 3, jj = i & 7;
    pp[head][ti][jj] = a.p[(uint64_t(start) + ti) * KC_HEADS * KC_RW + head * KC_RW + jj];
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncwarp();
  {
    const int ti = lane >> 2, head = lane & 3;
    if (ti < cnt) {
      float4 d4[KC_HEAD_DIM / 4];
#pragma unroll
      for (int m = 0; m < 8; m++) d4[m] = drows[lb_dout_f4(ti, head * 8 + m)];
      // s[j] = dOut_i · v_j: eight f64 chains side by side, each over d in order
      // (keys past the record read row 0 and are never used)
      A s[KC_RW];
#pragma unroll
      for (int j = 0; j < KC_RW; j++) s[j] = A(0);
#pragma unroll
      for (int m = 0; m < 8; m++)
#pragma unroll
        for (int j = 0; j < KC_RW; j++) {
          const float4 v = rows[la_exact_f4(j < cnt ? j : 0, 64 + head * 8 + m)];
          s[j] = fma(A(d4[m].x), A(v.x), s[j]);
          s[j] = fma(A(d4[m].y), A(v.y), s[j]);
          s[j] = fma(A(d4[m].z), A(v.z), s[j]);
          s[j] = fma(A(d4[m].w), A(v.w), s[j]);
        }
      A rs = A(0);
#pragma unroll
      for (int j = 0; j < KC_RW; j++)
        if (j < cnt) rs = rs + A(pp[head][ti][j]) * s[j];
#pragma unroll
      for (int j = 0; j < KC_RW; j++)
        if (j < cnt) dsh[head][ti][j] = f32(A(pp[head][ti][j]) * (A(f32(s[j])) - rs));
    }
  }
  __syncwarp();
  float* out = a.dqkv + uint64_t(start) * 3 * KC_H;
  const float* rowsf = reinterpret_cast<const float*>(rows);
  const float* drowsf = reinterpret_cast<const float*>(drows);
  // dQ_i = Σ_j dS_ij k_j, dK_i = Σ_j dS_ji q_j, dV_i = Σ_j P_ji dOut_j per
  // column: every row i of the record at once (24 f64 chains per lane), each
  // chain over j in order
  for (int m = 0; m < KC_HEADS; m++) {
    const int col = m * KC_HEAD_DIM + lane, f = m * 8 + (lane >> 2), c = lane & 3;
    A aq[KC_RW], ak[KC_RW], av[KC_RW];
#pragma unroll
    for (int i = 0; i < KC_RW; i++) aq[i] = ak[i] = av[i] = A(0);
#pragma unroll
    for (int j = 0; j < KC_RW; j++) {
      if (j >= cnt) break;
      const A kj = A(rowsf[la_exact_f4(j, 32 + f) * 4 + c]);
      const A qj = A(rowsf[la_exact_f4(j, f) * 4 + c]);
      const A dj = A(drowsf[lb_dout_f4(j, f) * 4 + c]);
#pragma unroll
      for (int i = 0; i < KC_RW; i++)
        if (i < cnt) {
          aq[i] = fma(A(dsh[m][i][j]), kj, aq[i]);
          ak[i] = fma(A(dsh[m][j][i]), qj, ak[i]);
          av[i] = fma(A(pp[m][j][i]), dj, av[i]);
        }
    }
#pragma unroll
    for (int i = 0; i < KC_RW; i++)
      if (i < cnt) {
        out[uint64_t(i) * 3 * KC_H + col] = f32(aq[i] * A(a.scale));
        out[uint64_t(i) * 3 * KC_H + KC_H + col] = f32(ak[i] * A(a.scale));
        out[uint64_t(i) * 3 * KC_H + 2 * KC_H + col] = f32(av[i]);
      }
  }
}

// learnFromExperience's per-frame readings (host/learn.ts:318-400), from a
// batch's backward: questions, bank rows, the critic's baseline (the mean of
// valuePrediction, summed in order), the value loss, and the report's
// entropy (Σ over rows with more than one allowed record of
// −Σ p·log p / log allowed, blocked = mask <= NEG_INF/2) and confidence
// (Σ p[target] over questions with a target row). One warp per frame; lane i
// walks question i (and i+32, ...), lane 0 adds the lanes' terms in question
// order.
constexpr int kLearnStats = 8;

__global__ void __launch_bounds__(256) k_learn_frame_stats(BatchGeo g, const float* p, const float* mask,
                                                          const float* pred, const double* loss,
                                                          const uint32_t* targets, uint32_t frames,
                                                          double* stats) {
  __shared__ double ent[8][32], conf[8][32];
  __shared__ int ent_ok[8][32], conf_ok[8][32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t f = blockIdx.x * 8 + warp;
  if (f >= frames) return;
  const uint64_t q0 = g.q_off[f], Q = g.q_off[f + 1] - q0;
  const uint64_t R = g.r_off[f + 1] - g.r_off[f], pb = g.p_off[f];
  double et = 0.0, er = 0.0, ct = 0.0, cr = 0.0;
  for (uint64_t base = 0; base < Q; base += 32) {
    const uint64_t i = base + lane;
    ent_ok[warp][lane] = 0;
    conf_ok[warp][lane] = 0;
    if (i < Q) {
      const float* prow = p + pb + i * R;
      const float* mrow = mask + pb + i * R;
      uint32_t allowed = 0;
      double e = 0.0;
      uint64_t j = 0;
      for (; j + 8 <= R; j += 8) {  // eight keys' loads in flight, the sum in key order
        float mv[8], pv[8];
#pragma unroll
        for (int u = 0; u < 8; u++) {
          mv[u] = mrow[j + u];
          pv[u] = prow[j + u];
        }
#pragma unroll
        for (int u = 0; u < 8; u++) {
          if (double(mv[u]) <= -1e30 / 2) continue;
          allowed++;
          const double pj = pv[u];
          if (pj > 0) e -= pj * log(pj);
        }
      }
      for (; j < R; j++) {
        if (double(mrow[j]) <= -1e30 / 2) continue;
        allowed++;
        const double pj = prow[j];
        if (pj > 0) e -= pj * log(pj);
      }
      if (allowed > 1) {
        ent[warp][lane] = e / log(double(allowed));
        ent_ok[warp][lane] = 1;
      }
      const uint32_t t = targets ? targets[q0 + i] : KC_INVALID;
      if (t != KC_INVALID && t < R) {
        conf[warp][lane] = prow[t];
        conf_ok[warp][lane] = 1;
      }
    }
    __syncwarp();
    if (lane == 0)
      for (int k = 0; k < 32; k++) {
        if (ent_ok[warp][k]) { et += ent[warp][k]; er += 1; }
        if (conf_ok[warp][k]) { ct += conf[warp][k]; cr += 1; }
      }
    __syncwarp();
  }
  if (lane == 0) {
    double baseline = 0.0;
    for (uint64_t i = 0; i < Q; i++) baseline += double(pred[q0 + i]);
    baseline = Q ? baseline / double(Q) : 0.0;
    double* o = stats + uint64_t(f) * kLearnStats;
    o[0] = double(Q); o[1] = double(R); o[2] = baseline; o[3] = loss[f];
    o[4] = et; o[5] = er; o[6] = ct; o[7] = cr;
  }
}

// The actor's and critic's batch gradients as the update applies them
// (host/learn.ts:440-470): out = [Σ_f step_f·dSelectorWq_f | Σ step_f·dSelectorWk_f
// | Σ step_f·dPool_f | Σ_f value_weight_f·dValueWv_f], in f64. Frames are
// summed in fixed chunks of kLearnChunk (partials [chunks][E]), then the
// chunks in order: deterministic for a given batch.
constexpr int kLearnChunk = 32;

__global__ void __launch_bounds__(256) k_learn_partial(const double* step, const double* value_weight,
                                                      const float* dwq, const float* dwk, const float* dpool,
                                                      const float* dwv, uint32_t frames, double* partial) {
  const uint32_t HH = KC_H * KC_H, E = 2 * HH + 2 * KC_H + 3 * KC_H;
  const uint32_t e = blockIdx.x * 256 + threadIdx.x;
  if (e >= E) return;
  const uint32_t f0 = blockIdx.y * kLearnChunk;
  const uint32_t f1 = f0 + kLearnChunk < frames ? f0 + kLearnChunk : frames;
  const float* src;
  uint32_t stride, off;
  const double* wgt = step;
  if (e < HH) { src = dwq; stride = HH; off = e; }
  else if (e < 2 * HH) { src = dwk; stride = HH; off = e - HH; }
  else if (e < 2 * HH + 2 * KC_H) { src = dpool; stride = 2 * KC_H; off = e - 2 * HH; }
  else { src = dwv; stride = 3 * KC_H; off = e - 2 * HH - 2 * KC_H; wgt = value_weight; }
  double acc = 0.0;
  for (uint32_t f = f0; f < f1; f++) {
    const double w = wgt[f];
    if (w != 0.0) acc += w * double(src[uint64_t(f) * stride + off]);
  }
  partial[uint64_t(blockIdx.y) * E + e] = acc;
}

__global__ void __launch_bounds__(256) k_learn_sum(const double* partial, uint32_t chunks, double* out) {
  const uint32_t E = 2 * KC_H * KC_H + 2 * KC_H + 3 * KC_H;
  const uint32_t e = blockIdx.x * 256 + threadIdx.x;
  if (e >= E) return;
  double acc = 0.0;
  for (uint32_t c = 0; c < chunks; c++) acc += partial[uint64_t(c) * E + e];
  out[e] = acc;
}

}  // namespace kc
