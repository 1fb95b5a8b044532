// exact.cuh — the forward in the reference oracle's exact arithmetic.
//
// Every kernel here reproduces packages/krystal/src/forward/oracle.ts the way
// JavaScript evaluates it: each dot product / weighted sum is ONE f64
// accumulator walked in the oracle's index order (products of two f32 are
// exact in f64, so an f64 FMA equals the oracle's multiply-then-add), and
// results are rounded to f32 exactly where the oracle stores into a
// Float32Array. Reductions whose order matters (softmax sums) are walked
// sequentially; order-free ones (max, any/all, first-argmax) run in parallel.
// The file is compiled with --fmad=false so that no a*b+c outside an
// explicit fma() is contracted.
#pragma once
#include "common.cuh"

namespace kc {

// ---------------------------------------------------------------------------
// fieldEmbed (oracle.ts:151-184): x[t] = token + field + schema + band +
// stream + pos rows, summed in that order in f64, stored f32 (H = 128).
// ---------------------------------------------------------------------------
struct EmbedArgs {
  const uint32_t* tok_recpos;
  const uint32_t* token_ids;
  const uint32_t* field_roles;
  const uint32_t* schema_ids;
  const uint32_t* band_ids;
  const uint32_t* token_rows;
  const float* table;  // embeddings page
  uint64_t tb_token, tb_field, tb_schema, tb_band, tb_stream, tb_pos;
  float* x;  // [T,128]
  uint64_t t;
  uint64_t small_floats;  // floats of the schema..pos tables staged in shared memory (0: read them from global)
};

// fieldEmbed (oracle.ts:151-184): x[t] = f32(token + field + schema + band +
// stream + pos rows, summed in that order in f64). A persistent grid of one
// CTA per SM. The CTA first stages the small tables in shared memory: the
// schema rows as f32, the band, stream and position rows already converted
// to f64 (the f32 -> f64 conversions, not the loads, bound this kernel), so
// that only the token and field rows are gathered from global memory (L2).
// Each warp takes 32 tokens at a time: lane i resolves token i's rows (the
// dependent chain record position -> token id -> tokenRows -> table row), so
// 32 chains are in flight at once; then the warp gathers the token and field
// rows of eight tokens at once and sums them with the staged rows, lane l
// owning columns 4l..4l+3.
constexpr int kEmbedWarps = 12;
constexpr int kEmbedTokensPerWarp = 32;
constexpr uint64_t kEmbedSmemMax = 200u << 10;

// Shared memory of k_embed_exact for the small tables (0: not staged).
__host__ __device__ inline uint64_t embed_smem_bytes(uint64_t schema_rows, uint64_t other_rows) {
  return schema_rows * KC_H * 4 + other_rows * KC_H * 8;
}

__global__ void __launch_bounds__(kEmbedWarps * 32, 1) k_embed_exact(EmbedArgs a) {
  extern __shared__ __align__(16) float emb_small[];
  // staged: schema rows (f32) | band, stream, pos rows (f64), contiguous in the page from tb_band
  const uint64_t n_schema = a.small_floats ? (a.tb_band - a.tb_schema) : 0;
  const uint64_t n_other = a.small_floats ? a.small_floats - n_schema : 0;
  double* emb_d = reinterpret_cast<double*>(emb_small + n_schema);
  for (uint64_t i = threadIdx.x; i < n_schema / 4; i += blockDim.x)
    reinterpret_cast<float4*>(emb_small)[i] = reinterpret_cast<const float4*>(a.table + a.tb_schema)[i];
  for (uint64_t i = threadIdx.x; i < n_other; i += blockDim.x) emb_d[i] = double(a.table[a.tb_band + i]);
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int d = lane * 4;
  const uint64_t stride = uint64_t(gridDim.x) * kEmbedWarps * kEmbedTokensPerWarp;
  for (uint64_t base = (uint64_t(blockIdx.x) * kEmbedWarps + warp) * kEmbedTokensPerWarp; base < a.t;
       base += stride) {
    const uint64_t left = a.t - base;
    const int n = left < kEmbedTokensPerWarp ? int(left) : kEmbedTokensPerWarp;
    uint32_t tok = 0, role = 0, schema = 0, band = 0, pos = 0;
    if (lane < n) {
      const uint32_t rp = a.tok_recpos[base + lane];
      const uint32_t g = rp >> 3;
      pos = rp & 7u;
      tok = a.token_rows[a.token_ids[uint64_t(g) * KC_RW + pos]];
      role = a.token_rows[a.field_roles[uint64_t(g) * KC_RW + pos]];
      schema = a.schema_ids[g];
      band = a.band_ids[g];
    }
    for (int i0 = 0; i0 < n; i0 += 8) {
      float4 r[8][2];
#pragma unroll
      for (int u = 0; u < 8; u++) {
        const int i = i0 + u;  // every lane shuffles; only tokens below n are read
        const uint32_t ti = __shfl_sync(0xffffffffu, tok, i & 31), ri = __shfl_sync(0xffffffffu, role, i & 31);
        if (i < n) {
          r[u][0] = *reinterpret_cast<const float4*>(a.table + a.tb_token + uint64_t(ti) * KC_H + d);
          r[u][1] = *reinterpret_cast<const float4*>(a.table + a.tb_field + uint64_t(ri) * KC_H + d);
        }
      }
#pragma unroll
      for (int u = 0; u < 8; u++) {
        const int i = i0 + u;
        const uint32_t si = __shfl_sync(0xffffffffu, schema, i & 31), bi = __shfl_sync(0xffffffffu, band, i & 31);
        const uint32_t li = __shfl_sync(0xffffffffu, pos, i & 31);
        if (i >= n) continue;
        const uint32_t stream = bi == KC_QUERY_BAND_ID ? 1u : 0u;
        const uint64_t ob = a.tb_band + uint64_t(bi) * KC_H + d, ost = a.tb_stream + uint64_t(stream) * KC_H + d;
        const uint64_t op = a.tb_pos + uint64_t(li) * KC_H + d, os = a.tb_schema + uint64_t(si) * KC_H + d;
        float4 s4;
        double b[4], st[4], p[4];
        if (n_other) {
          s4 = *reinterpret_cast<const float4*>(emb_small + (os - a.tb_schema));
          const double2* b2 = reinterpret_cast<const double2*>(emb_d + (ob - a.tb_band));
          const double2* st2 = reinterpret_cast<const double2*>(emb_d + (ost - a.tb_band));
          const double2* p2 = reinterpret_cast<const double2*>(emb_d + (op - a.tb_band));
          const double2 b01 = b2[0], b23 = b2[1], st01 = st2[0], st23 = st2[1], p01 = p2[0], p23 = p2[1];
          b[0] = b01.x; b[1] = b01.y; b[2] = b23.x; b[3] = b23.y;
          st[0] = st01.x; st[1] = st01.y; st[2] = st23.x; st[3] = st23.y;
          p[0] = p01.x; p[1] = p01.y; p[2] = p23.x; p[3] = p23.y;
        } else {
          s4 = *reinterpret_cast<const float4*>(a.table + os);
          const float4 b4 = *reinterpret_cast<const float4*>(a.table + ob);
          const float4 st4 = *reinterpret_cast<const float4*>(a.table + ost);
          const float4 p4 = *reinterpret_cast<const float4*>(a.table + op);
          b[0] = b4.x; b[1] = b4.y; b[2] = b4.z; b[3] = b4.w;
          st[0] = st4.x; st[1] = st4.y; st[2] = st4.z; st[3] = st4.w;
          p[0] = p4.x; p[1] = p4.y; p[2] = p4.z; p[3] = p4.w;
        }
        const float tv[4] = {r[u][0].x, r[u][0].y, r[u][0].z, r[u][0].w};
        const float fv[4] = {r[u][1].x, r[u][1].y, r[u][1].z, r[u][1].w};
        const float sv[4] = {s4.x, s4.y, s4.z, s4.w};
        float o[4];
#pragma unroll
        for (int e = 0; e < 4; e++) {
          double v = 0.0;
          v += double(tv[e]); v += double(fv[e]); v += double(sv[e]); v += b[e]; v += st[e]; v += p[e];
          o[e] = f32(v);
        }
        *reinterpret_cast<float4*>(a.x + (base + i) * KC_H + d) = make_float4(o[0], o[1], o[2], o[3]);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// matmulOracle (oracle.ts:114-125) and its fused consumers:
//   C = f32(A·Bᵀ)                          kEpiStore
//   C = relu(f32(A·Bᵀ))                    kEpiRelu   (reluOracle of the W1 output)
//   C = f32(C + f32(A·Bᵀ))                 kEpiResid  (addInPlace of the W2 output)
// A [M,K] f32, B [N,K] f32 (weights, [out,in]); every output is one f64
// accumulator over k = 0..K-1 in order. Square CTA tiles of 128, 64 or 32
// rows, operands converted to f64 once when staged in shared memory.
// Requires N % 128 == 0, K % 8 == 0, 16-byte aligned rows.
// ---------------------------------------------------------------------------
//   C = gate > 0 ? f32(A·Bᵀ) : 0            kEpiGate   (reluBackward of a saved ReLU output,
//                                                        backward.ts:65-70)
enum { kEpiStore = 0, kEpiRelu = 1, kEpiResid = 2, kEpiGate = 3 };

// BM x BM CTA tiles (BM = 128, 64 or 32) over 16 x 16 threads, each holding
// (BM/16)^2 accumulators at stride 16; the smaller tiles keep small-M
// products (mixer and selector rows of a few recomputed frames) spread over
// the SMs. The tiling never changes an output's accumulation order.
template <int EPI, int BM = 128>
__global__ void __launch_bounds__(256, BM == 128 ? 1 : 2) k_dgemm_exact(const float* __restrict__ A,
                                                                        const float* __restrict__ B, float* C, int M,
                                                                        int N, int K, int lda, int ldb, int ldc,
                                                                        const float* __restrict__ gate = nullptr) {
  constexpr int BN = BM, BK = 8, TM = BM / 16;
  __shared__ double As[2][BK][BM];
  __shared__ double Bs[2][BK][BN];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int64_t m0 = int64_t(blockIdx.x) * BM;  // row tiles on x: M may exceed 65535 tiles
  const int n0 = blockIdx.y * BN;
  const int lr = tid >> 1, lc = (tid & 1) * 4;
  const bool loader = lr < BM;  // thread lr stages row lr of the A and B tiles
  const bool a_ok = loader && m0 + lr < M;
  const float* Ap = A + (m0 + lr) * int64_t(lda) + lc;
  const float* Bp = B + int64_t(n0 + lr) * ldb + lc;

  double acc[TM][TM];
#pragma unroll
  for (int i = 0; i < TM; i++)
#pragma unroll
    for (int j = 0; j < TM; j++) acc[i][j] = 0.0;

  // a thread stages row lr of the A and B tiles, k-step s's four columns;
  // the global loads run two k-steps ahead of the products (registers x for
  // even steps, y for odd), so their latency spans two steps of DFMAs
  const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
  auto load_a = [&](int s) { return a_ok ? __ldg(reinterpret_cast<const float4*>(Ap + s * BK)) : z4; };
  auto load_b = [&](int s) { return loader ? __ldg(reinterpret_cast<const float4*>(Bp + s * BK)) : z4; };
  auto stage = [&](int buf, float4 ra, float4 rb) {
    if (!loader) return;
    As[buf][lc + 0][lr] = ra.x; As[buf][lc + 1][lr] = ra.y; As[buf][lc + 2][lr] = ra.z; As[buf][lc + 3][lr] = ra.w;
    Bs[buf][lc + 0][lr] = rb.x; Bs[buf][lc + 1][lr] = rb.y; Bs[buf][lc + 2][lr] = rb.z; Bs[buf][lc + 3][lr] = rb.w;
  };
  auto products = [&](int buf) {
#pragma unroll
    for (int kk = 0; kk < BK; kk++) {
      double av[TM], bv[TM];
#pragma unroll
      for (int i = 0; i < TM; i++) av[i] = As[buf][kk][ty + 16 * i];
#pragma unroll
      for (int j = 0; j < TM; j++) bv[j] = Bs[buf][kk][tx + 16 * j];
#pragma unroll
      for (int i = 0; i < TM; i++)
#pragma unroll
        for (int j = 0; j < TM; j++) acc[i][j] = fma(av[i], bv[j], acc[i][j]);
    }
  };
  const int steps = K / BK;
  float4 xa = load_a(0), xb = load_b(0), ya = z4, yb = z4;
  stage(0, xa, xb);
  if (steps > 1) { ya = load_a(1); yb = load_b(1); }
  __syncthreads();
  for (int s = 0; s < steps; s += 2) {
    if (s + 2 < steps) { xa = load_a(s + 2); xb = load_b(s + 2); }
    products(0);
    if (s + 1 < steps) stage(1, ya, yb);
    __syncthreads();
    if (s + 1 >= steps) break;
    if (s + 3 < steps) { ya = load_a(s + 3); yb = load_b(s + 3); }
    products(1);
    if (s + 2 < steps) stage(0, xa, xb);
    __syncthreads();
  }

#pragma unroll
  for (int i = 0; i < TM; i++) {
    const int64_t row = m0 + ty + 16 * i;
    if (row >= M) continue;
    float* cp = C + row * int64_t(ldc) + n0 + tx;
#pragma unroll
    for (int j = 0; j < TM; j++) {
      const float v = f32(acc[i][j]);
      if (EPI == kEpiStore) cp[16 * j] = v;
      else if (EPI == kEpiRelu) cp[16 * j] = js_relu(v);
      else if (EPI == kEpiGate) cp[16 * j] = gate[row * int64_t(ldc) + n0 + tx + 16 * j] > 0.0f ? v : 0.0f;
      else cp[16 * j] = f32(double(cp[16 * j]) + double(v));
    }
  }
}

// ---------------------------------------------------------------------------
// softmaxRow (oracle.ts:38-49) over a warp-held row of <= 8 f32 scores,
// evaluated by a single lane (the rows are at most 8 long).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void softmax_small(float* v, int count) {
  double mx = -INFINITY;
  for (int i = 0; i < count; i++) mx = js_max(mx, double(v[i]));
  double sum = 0.0;
  for (int i = 0; i < count; i++) {
    const double e = exp(double(v[i]) - mx);
    v[i] = f32(e);
    sum += e;
  }
  const double inv = 1.0 / js_max(sum, 1e-20);
  for (int i = 0; i < count; i++) v[i] = f32(double(v[i]) * inv);
}

// ---------------------------------------------------------------------------
// Record-local attention (attentionOracle local mode, oracle.ts:64-105, as
// called at :255) fused with the residual add (addInPlace, :256).
// One warp per record; lane = token*4 + head. q/k/v of the record are
// staged in shared memory; the head's output overwrites its q slice, then
// the warp adds the record's rows into x with coalesced stores.
// ---------------------------------------------------------------------------
struct LocalAttnArgs {
  const float* qkv;          // [T,384]: q | k | v
  float* x;                  // [T,128], updated in place
  const uint32_t* rec_start; // [N]
  const uint2* rec_meta;     // [N] (.y & 15 = token count)
  uint64_t records;
  double scale;              // 1/sqrt(headDim)
  float* p_out;              // optional [T][4][8]: the softmax row over the record's window
  const uint32_t* tok_recpos; // [T] record*8 | position, for the word ids
  const uint32_t* word_ids;   // optional [records*8]: the same-word bias's labels
  float word_alpha;           // the bias, f32 as the record mask stores it
};


// Staged q|k|v row r of a record: 96 float4 (q heads 0-3, k heads 4-7, v
// heads 8-11, 8 float4 each). Within each head's 8, float4 m sits at
// (m + 2·(head & 3) + (r & 1)) & 7, so the 8 lanes of a quarter-warp —
// heads 0-3 of two tokens — hit 8 different bank groups, reading q (one row
// each) or the same k / v row (4 distinct addresses).
__device__ __forceinline__ int la_exact_f4(int r, int f) {
  return r * 96 + (f & ~7) + (((f & 7) + 2 * ((f >> 3) & 3) + (r & 1)) & 7);
}

__global__ void __launch_bounds__(128) k_local_attn_exact(LocalAttnArgs a) {
  __shared__ float4 sm[4][KC_RW * 96];  // 48 KB
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint64_t g = uint64_t(blockIdx.x) * 4 + warp;
  if (g >= a.records) return;
  const uint32_t start = a.rec_start[g];
  const int cnt = int(a.rec_meta[g].y & 15u);
  if (cnt == 0) return;
  float4* rec = sm[warp];
  // stage q|k|v rows: cnt * 96 float4, every load in flight before the stores
  const float4* src = reinterpret_cast<const float4*>(a.qkv + uint64_t(start) * 3 * KC_H);
  for (int i = lane; i < cnt * 96; i += 32) cp_async16(rec + la_exact_f4(i / 96, i % 96), src + i);
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncwarp();
  const int ti = lane >> 2, head = lane & 3;
  float p[KC_RW];
  // word ids of the record's tokens: lane 4j holds token j's (all lanes shuffle)
  uint32_t wmine = KC_INVALID, wj[KC_RW];
  if (a.word_ids) {
    if (ti < cnt) wmine = a.word_ids[a.tok_recpos[start + ti]];
#pragma unroll
    for (int j = 0; j < KC_RW; j++) wj[j] = __shfl_sync(0xffffffffu, wmine, 4 * j);
  } else {
#pragma unroll
    for (int j = 0; j < KC_RW; j++) wj[j] = KC_INVALID;
  }
  float4 o4[KC_HEAD_DIM / 4];
  if (ti < cnt) {
    float4 q4[KC_HEAD_DIM / 4];
#pragma unroll
    for (int m = 0; m < 8; m++) q4[m] = rec[la_exact_f4(ti, head * 8 + m)];
    // the eight keys' f64 chains side by side, each over d = 0..31 in order
    // (keys past the record read row 0 and are never used)
    double s[KC_RW];
#pragma unroll
    for (int j = 0; j < KC_RW; j++) s[j] = 0.0;
#pragma unroll
    for (int m = 0; m < 8; m++)
#pragma unroll
      for (int j = 0; j < KC_RW; j++) {
        const float4 k = rec[la_exact_f4(j < cnt ? j : 0, (4 + head) * 8 + m)];
        s[j] = fma(double(q4[m].x), double(k.x), s[j]);
        s[j] = fma(double(q4[m].y), double(k.y), s[j]);
        s[j] = fma(double(q4[m].z), double(k.z), s[j]);
        s[j] = fma(double(q4[m].w), double(k.w), s[j]);
      }
#pragma unroll
    for (int j = 0; j < KC_RW; j++)
      if (j < cnt) p[j] = f32(s[j] * a.scale + double(word_bias(wmine, wj[j], a.word_alpha)));
    bool blocked = true;
    for (int j = 0; j < cnt; j++)
      if (double(p[j]) >= -1e29) { blocked = false; break; }
    if (blocked) {
      for (int j = 0; j < cnt; j++) p[j] = 0.0f;
    } else {
      softmax_small(p, cnt);
    }
    if (a.p_out)
      for (int j = 0; j < cnt; j++) a.p_out[((uint64_t(start) + ti) * KC_HEADS + head) * KC_RW + j] = p[j];
    // p·v: per output dimension an f64 chain over the record's keys in order
    double v[KC_HEAD_DIM];
#pragma unroll
    for (int d = 0; d < KC_HEAD_DIM; d++) v[d] = 0.0;
    for (int j = 0; j < cnt; j++) {
      const double pj = double(p[j]);
#pragma unroll
      for (int m = 0; m < 8; m++) {
        const float4 vv = rec[la_exact_f4(j, (8 + head) * 8 + m)];
        v[4 * m] = fma(pj, double(vv.x), v[4 * m]);
        v[4 * m + 1] = fma(pj, double(vv.y), v[4 * m + 1]);
        v[4 * m + 2] = fma(pj, double(vv.z), v[4 * m + 2]);
        v[4 * m + 3] = fma(pj, double(vv.w), v[4 * m + 3]);
      }
    }
#pragma unroll
    for (int m = 0; m < 8; m++) o4[m] = make_float4(f32(v[4 * m]), f32(v[4 * m + 1]), f32(v[4 * m + 2]), f32(v[4 * m + 3]));
  }
  __syncwarp();
  if (ti < cnt) {
    // every lane is done reading q (only lane ti*4+head reads this slice)
#pragma unroll
    for (int m = 0; m < 8; m++) rec[la_exact_f4(ti, head * 8 + m)] = o4[m];
  }
  __syncwarp();
  float4* xr = reinterpret_cast<float4*>(a.x + uint64_t(start) * KC_H);
  for (int i = lane; i < cnt * (KC_H / 4); i += 32) {
    const int r = i >> 5, f = i & 31;
    const float4 ov = rec[la_exact_f4(r, f)];
    float4 xv = xr[i];
    xv.x = f32(double(xv.x) + double(ov.x)); xv.y = f32(double(xv.y) + double(ov.y));
    xv.z = f32(double(xv.z) + double(ov.z)); xv.w = f32(double(xv.w) + double(ov.w));
    xr[i] = xv;
  }
}

// ---------------------------------------------------------------------------
// poolRecord (oracle.ts:186-224) for every record of the batch: two learned-
// query softmax poolings over the record's tokens. Bank records write their
// key and value rows; questions write their value row (the mixer's input
// state; the pooled query key is never read downstream).
// One warp per record.
// ---------------------------------------------------------------------------
struct PoolArgs {
  const float* x;            // [T,128]
  const float* pool;         // [2,128]
  const uint32_t* rec_start;
  const uint2* rec_meta;
  const uint32_t* rec_row;   // bank row, or question row | 0x80000000
  uint64_t records;
  double scale;              // 1/sqrt(H)
  float* bank_keys;          // [R,128]
  float* bank_values;        // [R,128]
  float* query_values;       // [Q,128]
};

__global__ void __launch_bounds__(256) k_pool_exact(PoolArgs a) {
  __shared__ float xs[8][KC_RW][KC_H];  // 32 KB
  __shared__ float ps[2][KC_H];
  __shared__ float sc[8][2][KC_RW];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < 2 * KC_H; i += 256) (&ps[0][0])[i] = a.pool[i];
  __syncthreads();
  const uint64_t g = uint64_t(blockIdx.x) * 8 + warp;
  if (g >= a.records) return;
  const uint32_t start = a.rec_start[g];
  const int cnt = int(a.rec_meta[g].y & 15u);
  const uint32_t row = a.rec_row[g];
  const bool isq = row & 0x80000000u;
  const uint32_t r = row & 0x7fffffffu;
  float* key_out = isq ? nullptr : a.bank_keys + uint64_t(r) * KC_H;
  float* val_out = isq ? a.query_values + uint64_t(r) * KC_H : a.bank_values + uint64_t(r) * KC_H;
  if (cnt == 0) {  // a record without tokens pools to zeros (oracle.ts:195)
    for (int d = lane; d < KC_H; d += 32) {
      if (key_out) key_out[d] = 0.0f;
      val_out[d] = 0.0f;
    }
    return;
  }
  const float4* src = reinterpret_cast<const float4*>(a.x + uint64_t(start) * KC_H);
  float4* dst = reinterpret_cast<float4*>(&xs[warp][0][0]);
  for (int i = lane; i < cnt * 32; i += 32) dst[i] = src[i];
  __syncwarp();
  // lanes 0..7: key scores, lanes 8..15: value scores
  if (lane < 16) {
    const int j = lane & 7, which = lane >> 3;
    if (j < cnt) {
      double s = 0.0;
      for (int d = 0; d < KC_H; d++) s = fma(double(ps[which][d]), double(xs[warp][j][d]), s);
      sc[warp][which][j] = f32(s * a.scale);
    }
  }
  __syncwarp();
  if (lane == 0 || lane == 8) softmax_small(sc[warp][lane >> 3], cnt);
  __syncwarp();
  for (int d = lane; d < KC_H; d += 32) {
    double ka = 0.0, va = 0.0;
    for (int j = 0; j < cnt; j++) {
      const double s = xs[warp][j][d];
      ka = fma(double(sc[warp][0][j]), s, ka);
      va = fma(double(sc[warp][1][j]), s, va);
    }
    if (key_out) key_out[d] = f32(ka);
    val_out[d] = f32(va);
  }
}

// Block-wide helpers for the per-question kernels (NT threads).
template <int NT>
__device__ __forceinline__ double block_js_max(double v, double* red) {
  for (int o = 16; o; o >>= 1) v = js_max(v, __shfl_xor_sync(0xffffffffu, v, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  double r = red[0];
  for (int w = 1; w < NT / 32; w++) r = js_max(r, red[w]);
  __syncthreads();
  return r;
}

template <int NT>
__device__ __forceinline__ int block_or(int v, int* red) {
  v = __any_sync(0xffffffffu, v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  int r = 0;
  for (int w = 0; w < NT / 32; w++) r |= red[w];
  __syncthreads();
  return r;
}

template <int NT>
__device__ __forceinline__ uint32_t block_sum_u32(uint32_t v, uint32_t* red) {
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  uint32_t r = 0;
  for (int w = 0; w < NT / 32; w++) r += red[w];
  __syncthreads();
  return r;
}

// ---------------------------------------------------------------------------
// Mixer cross-attention (attentionOracle dense mode with the session's open
// mixer mask, oracle.ts:292, session.ts:146) fused with the residual add
// (:293), in the oracle's arithmetic:
//   score_j = f32(Σ_d fma(q_d, k_jd) · scale + 0)   (f64, d in order)
//   m = max_j score_j;  e_j = exp(score_j − m) (f64)
//   sum = Σ_j e_j in index order (f64);  p_j = f32(f32(e_j) · (1 / max(sum, 1e-20)))
//   out_c = Σ_j fma(p_j, v_jc) in index order (f64);  x_c = f32(x_c + f32(out_c))
// with rows whose every score is below -1e29 giving p = 0.
//
// One CTA per chunk of up to QC (16, 8 or 4) questions of a frame, the chunks of a
// frame adjacent in the grid (they share the bank in L2). The bank's k rows
// stream through shared memory in blocks of kXaBlock keys, each loaded once
// for the whole chunk; three passes over the blocks compute the scores
// again, identically, each time: (1) the row maxima and the all-blocked test
// (neither depends on the order), (2) the exponentials, which one thread per
// row adds in index order, the sum carried from block to block, (3) p, then
// p·v, each output chain carried in index order from block to block.
//
// Score tiles: thread t takes head t>>6, questions 2((t&63)/G) and +1, keys
// ((t&63)%G) + G·i of the block (G = 64/(QC/2) key groups, i < QC/2); the k
// block's float4 c of row j sits at j*32 + (c ^ (j & 7)) so the 8 lanes of a
// quarter-warp read 8 bank groups. p·v tiles: thread t takes questions
// (QC/4)(t>>6) .. and columns 2(t&63), +1. A smaller chunk gives a batch of
// few frames more CTAs; the arithmetic of a question does not depend on it.
// ---------------------------------------------------------------------------
constexpr int kXaBlock = 64;
constexpr int kXaThreads = 256;
// k block f32 [kXaBlock][128] | q f64 [QC][128] | exponentials f64 [4 QC][kXaBlock] | p f32 [4 QC][kXaBlock]
constexpr size_t xa_smem(int qc) {
  return size_t(kXaBlock) * KC_H * 4 + size_t(qc) * KC_H * 8 + size_t(qc) * KC_HEADS * kXaBlock * 12;
}

struct CrossAttnArgs {
  const float* mq;          // [Q,128]
  const float* mk;          // [R,128]
  const float* mv;          // [R,128]
  float* query;             // [Q,128], updated in place
  const uint64_t* q_off;    // [frames + 1]
  const uint64_t* r_off;    // [frames + 1]
  int chunks;               // CTAs per frame: ceil(largest question count / the chunk)
  double scale;             // 1/sqrt(headDim)
  float* p_out;             // optional [4][sum Q_f R_f]: head h of question i at h*P + p_off[f] + il*R + j
  const uint64_t* p_off;
  uint64_t total_p;
};

template <int QC>
__global__ void __launch_bounds__(kXaThreads, 2) k_cross_attn_exact(CrossAttnArgs a) {
  constexpr int kRows = QC * KC_HEADS;
  constexpr int NK = QC / 2;          // keys per score thread
  constexpr int KG = kXaBlock / NK;   // key groups per (head, question pair)
  constexpr int PQ = QC / 4;          // questions per p·v thread
  extern __shared__ __align__(16) unsigned char dyn[];
  float4* ks = reinterpret_cast<float4*>(dyn);
  double* qd = reinterpret_cast<double*>(dyn + size_t(kXaBlock) * KC_H * 4);
  double* e64 = qd + QC * KC_H;
  float* pf = reinterpret_cast<float*>(e64 + kRows * kXaBlock);
  __shared__ double row_mx[kRows], row_inv[kRows];
  __shared__ int row_open[kRows];
  const uint32_t f = blockIdx.x / a.chunks;
  const int q0 = int(blockIdx.x % a.chunks) * QC;
  const uint64_t qb = a.q_off[f], rb = a.r_off[f];
  const int nq = int(a.q_off[f + 1] - qb), R = int(a.r_off[f + 1] - rb);
  if (q0 >= nq) return;
  const int nc = min(QC, nq - q0);
  const int tid = threadIdx.x;
  for (int i = tid; i < QC * KC_H; i += kXaThreads)
    qd[i] = i < nc * KC_H ? double(a.mq[(qb + q0) * KC_H + i]) : 0.0;
  const int nblk = (R + kXaBlock - 1) / kXaBlock;
  const float4* mk4 = reinterpret_cast<const float4*>(a.mk + rb * KC_H);
  auto stage = [&](int j0) {  // k rows [j0, j0 + block) into the block buffer
    const int nb = min(kXaBlock, R - j0);
    for (int i = tid; i < nb * 32; i += kXaThreads) {
      const int j = i >> 5, c4 = i & 31;
      cp_async16(ks + j * 32 + (c4 ^ (j & 7)), mk4 + size_t(j0 + j) * 32 + c4);
    }
  };
  auto staged = [&]() {
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();
  };

  const int s_head = tid >> 6, s_q = ((tid & 63) / KG) * 2, s_k = (tid & 63) % KG;
  // the tile's scores of the staged block (keys past its end are never used)
  auto scores = [&](float (&sf)[2][NK]) {
    double acc[2][NK];
#pragma unroll
    for (int c = 0; c < 2; c++)
#pragma unroll
      for (int i = 0; i < NK; i++) acc[c][i] = 0.0;
    const double* qp = qd + s_q * KC_H + s_head * KC_HEAD_DIM;
#pragma unroll 2
    for (int d4 = 0; d4 < (s_q < nc ? KC_HEAD_DIM / 4 : 0); d4++) {  // pairs past the chunk's questions: zeros
      float4 k4[NK];
#pragma unroll
      for (int i = 0; i < NK; i++) {
        const int j = s_k + KG * i;
        k4[i] = ks[j * 32 + ((s_head * 8 + d4) ^ (j & 7))];
      }
#pragma unroll
      for (int c = 0; c < 2; c++) {
        const double2 qa = *reinterpret_cast<const double2*>(qp + c * KC_H + 4 * d4);
        const double2 qc = *reinterpret_cast<const double2*>(qp + c * KC_H + 4 * d4 + 2);
#pragma unroll
        for (int i = 0; i < NK; i++) {
          acc[c][i] = fma(qa.x, double(k4[i].x), acc[c][i]);
          acc[c][i] = fma(qa.y, double(k4[i].y), acc[c][i]);
          acc[c][i] = fma(qc.x, double(k4[i].z), acc[c][i]);
          acc[c][i] = fma(qc.y, double(k4[i].w), acc[c][i]);
        }
      }
    }
#pragma unroll
    for (int c = 0; c < 2; c++)
#pragma unroll
      for (int i = 0; i < NK; i++) sf[c][i] = f32(acc[c][i] * a.scale + 0.0);
  };
  const int row0 = s_q * KC_HEADS + s_head;  // the tile's rows: row0 and row0 + 4

  // (1) row maxima and the all-blocked test
  {
    double m[2] = {-INFINITY, -INFINITY};
    bool open[2] = {false, false};
    if (nblk > 0) stage(0);
    for (int b = 0; b < nblk; b++) {
      const int j0 = b * kXaBlock, nb = min(kXaBlock, R - j0);
      staged();
      float sf[2][NK];
      scores(sf);
      __syncthreads();
      if (b + 1 < nblk) stage(j0 + kXaBlock);
#pragma unroll
      for (int c = 0; c < 2; c++)
#pragma unroll
        for (int i = 0; i < NK; i++)
          if (s_k + KG * i < nb) {
            m[c] = js_max(m[c], double(sf[c][i]));
            open[c] |= double(sf[c][i]) >= -1e29;
          }
    }
#pragma unroll
    for (int c = 0; c < 2; c++) {
      for (int o = 1; o < KG; o <<= 1) {
        m[c] = js_max(m[c], __shfl_xor_sync(0xffffffffu, m[c], o));
        open[c] |= __shfl_xor_sync(0xffffffffu, int(open[c]), o) != 0;
      }
      if (s_k == 0) {
        row_mx[row0 + 4 * c] = m[c];
        row_open[row0 + 4 * c] = open[c];
      }
    }
  }
  __syncthreads();
  const double mx0 = row_mx[row0], mx1 = row_mx[row0 + 4];
  const bool op0 = row_open[row0] != 0, op1 = row_open[row0 + 4] != 0;

  // (2) exponentials; thread r < kRows adds row r's in index order
  {
    double sum = 0.0;
    const bool summer = tid < kRows && row_open[tid] != 0;
    if (nblk > 0) stage(0);
    for (int b = 0; b < nblk; b++) {
      const int j0 = b * kXaBlock, nb = min(kXaBlock, R - j0);
      staged();
      float sf[2][NK];
      scores(sf);
#pragma unroll
      for (int i = 0; i < NK; i++) {
        const int j = s_k + KG * i;
        if (j < nb) {
          if (op0) e64[row0 * kXaBlock + j] = exp(double(sf[0][i]) - mx0);
          if (op1) e64[(row0 + 4) * kXaBlock + j] = exp(double(sf[1][i]) - mx1);
        }
      }
      __syncthreads();
      if (b + 1 < nblk) stage(j0 + kXaBlock);
      if (summer)
        for (int j = 0; j < nb; j++) sum += e64[tid * kXaBlock + j];
    }
    if (tid < kRows) row_inv[tid] = 1.0 / js_max(sum, 1e-20);
  }
  __syncthreads();
  const double inv0 = row_inv[row0], inv1 = row_inv[row0 + 4];

  // (3) p, then p·v
  const int v_q = (tid >> 6) * PQ, v_col = (tid & 63) * 2, v_head = (tid & 63) >> 4;
  double acc[PQ][2];
#pragma unroll
  for (int c = 0; c < PQ; c++) acc[c][0] = acc[c][1] = 0.0;
  if (nblk > 0) stage(0);
  for (int b = 0; b < nblk; b++) {
    const int j0 = b * kXaBlock, nb = min(kXaBlock, R - j0);
    staged();
    {
      float sf[2][NK];
      scores(sf);
#pragma unroll
      for (int i = 0; i < NK; i++) {
        const int j = s_k + KG * i;
        if (j < nb) {
          const float p0 = op0 ? f32(double(f32(exp(double(sf[0][i]) - mx0))) * inv0) : 0.0f;
          const float p1 = op1 ? f32(double(f32(exp(double(sf[1][i]) - mx1))) * inv1) : 0.0f;
          pf[row0 * kXaBlock + j] = p0;
          pf[(row0 + 4) * kXaBlock + j] = p1;
          if (a.p_out) {
            const uint64_t base = uint64_t(s_head) * a.total_p + a.p_off[f] + uint64_t(j0 + j);
            if (s_q < nc) a.p_out[base + uint64_t(q0 + s_q) * R] = p0;
            if (s_q + 1 < nc) a.p_out[base + uint64_t(q0 + s_q + 1) * R] = p1;
          }
        }
      }
    }
    __syncthreads();
    if (b + 1 < nblk) stage(j0 + kXaBlock);
    if (v_q < nc) {
      const float* pr = pf + (v_q * KC_HEADS + v_head) * kXaBlock;
      const float* vr = a.mv + (rb + j0) * KC_H + v_col;
      int j = 0;
      for (; j + 4 <= nb; j += 4) {
        float2 v[4];
#pragma unroll
        for (int u = 0; u < 4; u++) v[u] = *reinterpret_cast<const float2*>(vr + size_t(j + u) * KC_H);
#pragma unroll
        for (int c = 0; c < PQ; c++) {
          const float4 p4 = *reinterpret_cast<const float4*>(pr + c * KC_HEADS * kXaBlock + j);
          const float pv[4] = {p4.x, p4.y, p4.z, p4.w};
#pragma unroll
          for (int u = 0; u < 4; u++) {
            acc[c][0] = fma(double(pv[u]), double(v[u].x), acc[c][0]);
            acc[c][1] = fma(double(pv[u]), double(v[u].y), acc[c][1]);
          }
        }
      }
      for (; j < nb; j++) {
        const float2 v = *reinterpret_cast<const float2*>(vr + size_t(j) * KC_H);
#pragma unroll
        for (int c = 0; c < PQ; c++) {
          const double pj = double(pr[c * KC_HEADS * kXaBlock + j]);
          acc[c][0] = fma(pj, double(v.x), acc[c][0]);
          acc[c][1] = fma(pj, double(v.y), acc[c][1]);
        }
      }
    }
  }
#pragma unroll
  for (int c = 0; c < PQ; c++)
    if (v_q + c < nc) {
      float* qp = a.query + (qb + q0 + v_q + c) * KC_H + v_col;
      qp[0] = f32(double(qp[0]) + double(f32(acc[c][0])));
      qp[1] = f32(double(qp[1]) + double(f32(acc[c][1])));
    }
}

// ---------------------------------------------------------------------------
// selectorOracle (oracle.ts:332-382) for one question per CTA:
// score = f32(qProj·kProj · (1/sqrt(H)) + mask), all-blocked rows -> p = 0 and
// KC_NO_SELECTION, softmaxRow, first-max argmax over the stored p (or
// sampleRow, sampling.ts:41-57), optional soft gather.
// The mask is the open mask, an explicit [Q,R] mask, or the rule form of
// selectionMask (host/learn.ts:215-232) with reopen-if-none-admitted (:229).
// ---------------------------------------------------------------------------
struct SelectArgs {
  const float* sq;          // [Q,128] query projections
  const float* sk;          // [R,128] bank key projections
  const float* bank_values; // [R,128], for the gather (may be null)
  const uint32_t* query_frame;
  const uint64_t* r_off;
  const uint64_t* q_off;
  const uint64_t* p_off;
  const float* mask;        // explicit mask laid out like p, or null
  const uint32_t* schema_allow; // rule, or null
  const uint32_t* band_allow;
  const uint32_t* bank_rec;  // bank row -> record (for the rule)
  const uint32_t* schema_ids;
  const uint32_t* band_ids;
  const double* uniforms;   // [Q] or null
  uint32_t max_r;
  double scale;             // 1/sqrt(H)
  float* p;                 // [sum Q_f R_f]
  uint32_t* index;          // [Q]
  float* gather;            // [Q,128] or null
};

// selectorOracle's masked scores (oracle.ts:340-345) for a chunk of up to
// kXsChunk questions of a frame per CTA, the chunks of a frame adjacent in the
// grid: score_j = f32(Σ_d fma(q_d, k_jd) · scale + mask_j) with the f64 chain
// in dimension order, written into the question's p row for k_select_exact
// to finish. The bank's key rows stream through shared memory in blocks of
// kXsBlock, each loaded once for the chunk (float4 c of row j at
// j*32 + (c ^ (j & 7))); warp w takes questions 2w and 2w+1, lane l the keys
// l and l+32 of the block. The rule mask's reopen-if-none-admitted
// (host/learn.ts:229) is counted first for each question.
constexpr int kXsChunk = 16;
constexpr int kXsBlock = 64;
constexpr int kXsThreads = 256;
constexpr size_t kXsSmem = size_t(kXsBlock) * KC_H * 4 + size_t(kXsChunk) * KC_H * 8;

__global__ void __launch_bounds__(kXsThreads) k_select_scores_exact(SelectArgs a, int chunks) {
  extern __shared__ __align__(16) unsigned char dyn[];
  float4* ks = reinterpret_cast<float4*>(dyn);
  double* qd = reinterpret_cast<double*>(dyn + size_t(kXsBlock) * KC_H * 4);
  __shared__ uint32_t s_allow[kXsChunk][9];  // schema words 0-7, band word 8
  __shared__ uint32_t s_admitted[kXsChunk];
  __shared__ uint32_t s_rec[kXsBlock];       // the block's keys: schema | band << 16, or ~0 when out of range
  const uint32_t f = blockIdx.x / chunks;
  const int q0 = int(blockIdx.x % chunks) * kXsChunk;
  const uint64_t qb = a.q_off[f], rb = a.r_off[f];
  const int nq = int(a.q_off[f + 1] - qb), R = int(a.r_off[f + 1] - rb);
  if (q0 >= nq || R == 0) return;
  const int nc = min(kXsChunk, nq - q0);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int i = tid; i < kXsChunk * KC_H; i += kXsThreads)
    qd[i] = i < nc * KC_H ? double(a.sq[(qb + q0) * KC_H + i]) : 0.0;
  const bool rule = a.mask == nullptr && a.schema_allow != nullptr;
  auto key_ok = [&](int c, uint32_t sb) {
    const uint32_t sid = sb & 0xffffu, b = sb >> 16;
    return sid < 256u && b < 32u && ((s_allow[c][sid >> 5] >> (sid & 31)) & 1u) && ((s_allow[c][8] >> b) & 1u);
  };
  auto rec_of = [&](int j) {  // schema | band << 16 of bank row j (ids >= 65536 read as out of range)
    const uint32_t g = a.bank_rec[rb + j];
    const uint32_t sid = a.schema_ids[g], b = a.band_ids[g];
    return (sid < 65536u && b < 65536u) ? (sid | (b << 16)) : 0xffffffffu;
  };
  if (rule) {
    for (int i = tid; i < kXsChunk * 9; i += kXsThreads) {
      const int c = i / 9, w = i % 9;
      s_allow[c][w] = c < nc ? (w < 8 ? a.schema_allow[(qb + q0 + c) * 8 + w] : a.band_allow[qb + q0 + c]) : 0u;
    }
    if (tid < kXsChunk) s_admitted[tid] = 0;
    __syncthreads();
    uint32_t cnt[kXsChunk];
#pragma unroll
    for (int c = 0; c < kXsChunk; c++) cnt[c] = 0;
    for (int j = tid; j < R; j += kXsThreads) {
      const uint32_t sb = rec_of(j);
#pragma unroll
      for (int c = 0; c < kXsChunk; c++) cnt[c] += key_ok(c, sb) ? 1u : 0u;
    }
#pragma unroll
    for (int c = 0; c < kXsChunk; c++)
      if (c < nc && cnt[c]) atomicAdd(&s_admitted[c], cnt[c]);
  }
  const int nblk = (R + kXsBlock - 1) / kXsBlock;
  const float4* sk4 = reinterpret_cast<const float4*>(a.sk + rb * KC_H);
  auto stage = [&](int j0) {
    const int nb = min(kXsBlock, R - j0);
    for (int i = tid; i < nb * 32; i += kXsThreads) {
      const int j = i >> 5, c4 = i & 31;
      cp_async16(ks + j * 32 + (c4 ^ (j & 7)), sk4 + size_t(j0 + j) * 32 + c4);
    }
  };
  const int c0 = warp * 2;
  stage(0);
  for (int b = 0; b < nblk; b++) {
    const int j0 = b * kXsBlock, nb = min(kXsBlock, R - j0);
    if (rule && tid < kXsBlock) s_rec[tid] = tid < nb ? rec_of(j0 + tid) : 0xffffffffu;
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();
    double acc[2][2] = {{0.0, 0.0}, {0.0, 0.0}};
    if (c0 < nc) {
      const double* qp = qd + c0 * KC_H;
#pragma unroll 4
      for (int d4 = 0; d4 < KC_H / 4; d4++) {
        float4 k4[2];
#pragma unroll
        for (int t = 0; t < 2; t++) {
          const int j = lane + 32 * t;
          k4[t] = ks[j * 32 + (d4 ^ (j & 7))];
        }
#pragma unroll
        for (int c = 0; c < 2; c++) {
          const double2 qa = *reinterpret_cast<const double2*>(qp + c * KC_H + 4 * d4);
          const double2 qc = *reinterpret_cast<const double2*>(qp + c * KC_H + 4 * d4 + 2);
#pragma unroll
          for (int t = 0; t < 2; t++) {
            acc[c][t] = fma(qa.x, double(k4[t].x), acc[c][t]);
            acc[c][t] = fma(qa.y, double(k4[t].y), acc[c][t]);
            acc[c][t] = fma(qc.x, double(k4[t].z), acc[c][t]);
            acc[c][t] = fma(qc.y, double(k4[t].w), acc[c][t]);
          }
        }
      }
#pragma unroll
      for (int c = 0; c < 2; c++) {
        const int qi = q0 + c0 + c;
        if (c0 + c >= nc) continue;
        float* prow = a.p + a.p_off[f] + uint64_t(qi) * R + j0;
        const bool reopen = rule && s_admitted[c0 + c] == 0;
#pragma unroll
        for (int t = 0; t < 2; t++) {
          const int j = lane + 32 * t;
          if (j >= nb) continue;
          float m = 0.0f;
          if (a.mask) m = a.mask[a.p_off[f] + uint64_t(qi) * R + j0 + j];
          else if (rule && !reopen) m = key_ok(c0 + c, s_rec[j]) ? 0.0f : -1e30f;
          prow[j] = f32(acc[c][t] * a.scale + double(m));
        }
      }
    }
    __syncthreads();
    if (b + 1 < nblk) stage(j0 + kXsBlock);
  }
}

// The rest of selectorOracle for one question per CTA, from the masked
// scores k_select_scores_exact left in the question's p row:
__global__ void __launch_bounds__(256) k_select_exact(SelectArgs a) {
  constexpr int NT = 256;
  extern __shared__ __align__(16) unsigned char dyn[];
  __shared__ double red[NT / 32];
  __shared__ int redi[NT / 32];
  __shared__ double inv_s;
  __shared__ float bestv[NT / 32];
  __shared__ uint32_t besti[NT / 32];
  const uint32_t qi = blockIdx.x;
  const uint32_t f = a.query_frame[qi];
  const uint64_t rb = a.r_off[f];
  const int R = int(a.r_off[f + 1] - rb);
  const uint64_t il = qi - a.q_off[f];  // question index within the frame
  float* prow = a.p + a.p_off[f] + il * uint64_t(R);
  if (R == 0) {
    if (threadIdx.x == 0) a.index[qi] = KC_INVALID;
    return;
  }
  double* e64 = reinterpret_cast<double*>(dyn);               // [max_r]
  float* sc = reinterpret_cast<float*>(e64 + size_t(a.max_r)); // [max_r]
  const int tid = threadIdx.x;
  for (int j = tid; j < R; j += NT) sc[j] = prow[j];
  __syncthreads();

  // scores.every(score => score < -1e29): NaN is NOT blocked here
  int open = 0;
  double mx = -INFINITY;
  for (int j = tid; j < R; j += NT) {
    open |= !(double(sc[j]) < -1e29);
    mx = js_max(mx, double(sc[j]));
  }
  const bool all_blocked = !block_or<NT>(open, redi);
  if (all_blocked) {
    for (int j = tid; j < R; j += NT) sc[j] = 0.0f;
  } else {
    mx = block_js_max<NT>(mx, red);
    for (int j = tid; j < R; j += NT) {
      const double e = exp(double(sc[j]) - mx);
      e64[j] = e;
      sc[j] = f32(e);
    }
    __syncthreads();
    if (tid == 0) {
      double sum = 0.0;
      for (int j = 0; j < R; j++) sum += e64[j];
      inv_s = 1.0 / js_max(sum, 1e-20);
    }
    __syncthreads();
    const double inv = inv_s;
    for (int j = tid; j < R; j += NT) sc[j] = f32(double(sc[j]) * inv);
  }
  __syncthreads();
  for (int j = tid; j < R; j += NT) prow[j] = sc[j];

  // first j with the largest p (strict > scan from best = 0, oracle.ts:359-363):
  // the first index of the maximum over non-NaN p, unless p[0] is NaN.
  float bv = -INFINITY;
  uint32_t bi = KC_INVALID;
  for (int j = tid; j < R; j += NT) {
    const float v = sc[j];
    if (v == v && (bi == KC_INVALID || v > bv)) { bv = v; bi = uint32_t(j); }
  }
  for (int o = 16; o; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (oi != KC_INVALID && (bi == KC_INVALID || ov > bv || (ov == bv && oi < bi))) { bv = ov; bi = oi; }
  }
  if ((tid & 31) == 0) { bestv[tid >> 5] = bv; besti[tid >> 5] = bi; }
  __syncthreads();
  if (tid == 0) {
    float v = bestv[0];
    uint32_t b = besti[0];
    for (int w = 1; w < NT / 32; w++) {
      const float ov = bestv[w];
      const uint32_t oi = besti[w];
      if (oi != KC_INVALID && (b == KC_INVALID || ov > v || (ov == v && oi < b))) { v = ov; b = oi; }
    }
    uint32_t best = (sc[0] != sc[0] || b == KC_INVALID) ? 0u : b;
    if (all_blocked) {
      best = KC_INVALID;
    } else if (a.uniforms) {  // sampleRow (sampling.ts:41-57)
      const double u = a.uniforms[qi];
      double cum = 0.0;
      int last = -1, drawn = -2;
      for (int j = 0; j < R; j++) {
        const double w = sc[j];
        if (!(w > 0)) continue;
        last = j;
        cum += w;
        if (u < cum) { drawn = j; break; }
      }
      if (drawn == -2) drawn = last;
      best = drawn < 0 ? KC_INVALID : uint32_t(drawn);
    }
    a.index[qi] = best;
  }
  if (a.gather) {
    for (int d = tid; d < KC_H; d += NT) {
      double g = 0.0;
      for (int j = 0; j < R; j++) g = fma(double(sc[j]), double(a.bank_values[(rb + j) * KC_H + d]), g);
      a.gather[uint64_t(qi) * KC_H + d] = f32(g);
    }
  }
}

}  // namespace kc
