// krystal_cuda.cu — the C ABI (include/krystal_cuda.h) and the batch driver.
//
// One handle = one device, one stream, one device copy of the weight page,
// and a grow-only workspace sized to the largest batch seen. A batch runs as:
//
//   pack      k_frame_scan -> k_frame_offsets -> (one 64-byte readback of the
//             batch totals, the only host wait) -> k_record_rows
//   embed     k_embed_exact                                 fieldEmbed
//   encoder   per block: QKV GEMM, local attention + residual,
//             W1 GEMM + ReLU, W2 GEMM + residual            oracle.ts:250-259
//   pool      k_pool_exact                                  oracle.ts:261-283
//   mixer     per block: Q/K/V GEMMs, cross-attention + residual,
//             W1 GEMM + ReLU, W2 GEMM + residual            oracle.ts:285-296
//   selector  Wq/Wk GEMMs, k_select_exact                   oracle.ts:332-382
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cstdlib>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/krystal_cuda.h"
#include "backward.cuh"
#include "common.cuh"
#include "exact.cuh"
#include "fast.cuh"
#include "ffn.cuh"
#include "attn_tc.cuh"
#include "learn.cuh"
#include "ozaki.cuh"
#include "pack.cuh"
#include "tc_gemm.cuh"

namespace {

thread_local std::string g_create_error;

// A grow-only device buffer; it frees its memory when its owner is destroyed.
struct DevBuf {
  void* p = nullptr;
  size_t cap = 0;
  DevBuf() = default;
  DevBuf(const DevBuf&) = delete;
  DevBuf& operator=(const DevBuf&) = delete;
  ~DevBuf() {
    if (p) cudaFree(p);
  }
};

double now_ms() {
  return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

// Workspace reallocations made by this thread, and the time they took (a
// cudaFree waits for the device): the stream's worker reports them per batch.
thread_local uint64_t t_grows = 0;
thread_local double t_grow_ms = 0;

template <typename T>
T* P(DevBuf& b) { return static_cast<T*>(b.p); }

struct Dims {
  uint32_t h, heads, hd, ffn, enc, mix, route;
  uint32_t token_space, field_space, schema_space, band_space, stream_space, pos_space;
  uint64_t tb_token, tb_field, tb_schema, tb_band, tb_stream, tb_pos;
  uint64_t emb_elems, off_enc, off_pool, off_mixer, off_swq, off_swk, off_dec, off_val, total, block;
};

Dims dims_of(const kc_config* c) {
  Dims d{};
  d.h = c->hidden_size; d.heads = c->head_count; d.hd = c->head_dim; d.ffn = c->ffn_size;
  d.enc = c->encoder_blocks; d.mix = c->mixer_blocks; d.route = c->route_kind_count;
  d.token_space = c->token_space; d.field_space = c->field_space; d.schema_space = c->schema_space;
  d.band_space = c->band_space; d.stream_space = c->stream_space; d.pos_space = c->pos_space;
  const uint64_t h = d.h, f = d.ffn;
  uint64_t cur = 0;
  d.tb_token = cur; cur += uint64_t(d.token_space) * h;
  d.tb_field = cur; cur += uint64_t(d.field_space) * h;
  d.tb_schema = cur; cur += uint64_t(d.schema_space) * h;
  d.tb_band = cur; cur += uint64_t(d.band_space) * h;
  d.tb_stream = cur; cur += uint64_t(d.stream_space) * h;
  d.tb_pos = cur; cur += uint64_t(d.pos_space) * h;
  d.emb_elems = cur;
  d.block = 3 * h * h + 2 * f * h;
  d.off_enc = cur; cur += d.block * d.enc;
  d.off_pool = cur; cur += 2 * h;
  d.off_mixer = cur; cur += d.block * d.mix;
  d.off_swq = cur; cur += h * h;
  d.off_swk = cur; cur += h * h;
  d.off_dec = cur; cur += uint64_t(d.route) * 3 * h;
  d.off_val = cur; cur += 3 * h;
  d.total = cur;
  return d;
}

struct Workspace {
  // staged inputs (host entry points)
  DevBuf rec_off, token_ids, field_roles, schema_ids, band_ids, schema_allow, band_allow, uniforms, mask;
  DevBuf word_ids;
  DevBuf bank_schema, bank_band;
  // pack
  DevBuf rec_meta, frame_t, frame_q, frame_r, t_off, q_off, r_off, p_off, totals;
  DevBuf tok_recpos, rec_start, rec_row, bank_rec, bank_frame, query_rec, query_frame;
  // the fused attention's record-aligned tiles (first row per tile) and row info
  DevBuf tile_row, row_rc;
  // activations
  DevBuf x, qkv, bk, bv, mk, mv, qstate, mq, mh, sq, sk, p, index, gather;
  // weight-row scatter staging
  DevBuf rows_val, rows_off;
  // certification flags per frame, and the list of frames to recompute
  DevBuf flags, list;
  // the certificate's inputs: |sq|, |sk| per row and kappa_q per question
  DevBuf nq, nk, kappa;
};

// The backward's buffers: what the forward saves for it (per block), the
// request, the intermediate gradients, and the per-frame results.
struct BackWs {
  DevBuf mask, targets, valence;
  DevBuf enc_qkv, enc_p, enc_h1, mix_q, mix_k, mix_v, mix_p, mix_h1;
  DevBuf gather, offered, n_allowed, pred, dpred, loss, dwv;
  DevBuf dquery, dig, dag, dscore, dqp, dkp, dbk, dbv, dswq, dswk;
  DevBuf dh1, ads, mdq, mdk, mdv, tok_ds, dfs, dpool, edqkv;
  DevBuf learn_partial;
  // the device learn step's rollback copy, health words and readback
  DevBuf learn_backup, learn_health, learn_out;
  // the last batch differentiated: its frame count and the selection it ran under
  uint32_t frames = 0;
  const float* mask_used = nullptr;
};

enum Stage { kStPack, kStEmbed, kStEncGemm, kStEncAttn, kStPool, kStMixer, kStSelector, kStFallback, kStEncFfn,
             kStEncAttnTc, kStCount };

// The matrices the tensor-core path multiplies by, in a fixed order:
// per encoder block QKV [3H,H], W1 [F,H], W2 [H,F]; per mixer block Wq, Wk,
// Wv [H,H], W1, W2; the selector's Wq, Wk. Then the same list again,
// transposed (the backward's input products): entry nF + i is the transpose
// of entry i, read from the transposed page, where an encoder block's QKV
// becomes one [H, 3H] matrix [Wqᵀ | Wkᵀ | Wvᵀ].
struct Mat {
  uint64_t page_off;
  uint32_t n, k;
  bool transposed;
};

std::vector<Mat> mat_list(const Dims& d) {
  std::vector<Mat> v;
  const uint64_t hh = uint64_t(d.h) * d.h, fh = uint64_t(d.ffn) * d.h;
  for (int t = 0; t < 2; t++) {
    const bool tr = t == 1;
    auto add = [&](uint64_t off, uint32_t n, uint32_t k) { v.push_back(tr ? Mat{off, k, n, true} : Mat{off, n, k, false}); };
    for (uint32_t b = 0; b < d.enc; b++) {
      const uint64_t o = d.off_enc + d.block * b;
      add(o, 3 * d.h, d.h);
      add(o + 3 * hh, d.ffn, d.h);
      add(o + 3 * hh + fh, d.h, d.ffn);
    }
    for (uint32_t b = 0; b < d.mix; b++) {
      const uint64_t o = d.off_mixer + d.block * b;
      add(o, d.h, d.h);
      add(o + hh, d.h, d.h);
      add(o + 2 * hh, d.h, d.h);
      add(o + 3 * hh, d.ffn, d.h);
      add(o + 3 * hh + fh, d.h, d.ffn);
    }
    add(d.off_swq, d.h, d.h);
    add(d.off_swk, d.h, d.h);
  }
  return v;
}

}  // namespace

struct kc_handle {
  std::mutex mu;
  int device = 0;
  int sms = 148;
  cudaStream_t own = nullptr;
  cudaStream_t stream = nullptr;
  Dims d{};
  float* w = nullptr;
  uint32_t* token_rows = nullptr;
  uint32_t token_rows_len = 0;
  std::vector<uint32_t> token_rows_host;  // for validating frames on the host (streams)
  std::vector<uint8_t> id_ok;             // per id: bit 0 a valid token, bit 1 a valid field role
  Workspace ws;      // the batch
  Workspace ws_fb;   // frames recomputed on the exact path
  BackWs bw;         // the backward
  DevBuf wt;         // transposed copies of the block and selector matrices (page layout)
  bool wt_blocks_dirty = true;  // the blocks' transposed copies are stale
  bool wt_sel_dirty = true;     // the selector's transposed copies are stale
  kc::FrameTotals* h_tot = nullptr;  // pinned
  std::string err;
  uint64_t launches = 0;
  // the batch whose encodings are resident in ws for kc_select_batch: ws_epoch
  // counts packings into ws and weight changes; the batch is resident while
  // resident_epoch still equals it
  uint64_t ws_epoch = 0, resident_epoch = 0;
  int resident_precision = KC_PRECISION_CERTIFIED;
  uint32_t resident_frames = 0;
  uint64_t resident_records = 0;
  float resident_alpha = 0.0f;      // the resident batch's same-word bias (its ids stay in ws.word_ids)
  bool resident_words = false;
  kc::FrameTotals resident_tot{};   // the resident batch's totals
  bool last_overflow = false;       // the last certified batch split out of range
  // the fused encoder kernels (k_tc_attn, k_tc_ffn) where the dimensions fit;
  // KC_NO_FUSION=1 in the environment at kc_create runs the unfused sequence
  // (the same arithmetic, kept for the learn path and checked against the fused)
  bool fuse = true;
  // the exact path's GEMMs on the int8 tensor cores (ozaki.cuh), with the
  // FP64 kernel's results; KC_NO_OZAKI=1 at kc_create keeps them on the FP64
  // kernel. oz_suspend runs a forward again on the FP64 kernel after a list
  // overflow.
  bool oz = true, oz_suspend = false, oz_ran = false;
  long long oz_cap = -1;            // KC_OZAKI_LIST_CAP at kc_create: the list's length (tests); -1 sized by M·N
  DevBuf oz_w;                      // weight slices and row data per forward matrix
  std::vector<uint64_t> oz_w_off;   // per matrix (forward ones only): offset into oz_w
  std::vector<char> oz_dirty;       // per matrix: its slices are stale
  DevBuf oz_a, oz_meta, oz_list;    // A slices, A row data, the listed outputs
  unsigned* d_oz_word = nullptr;    // [0] listed outputs of the current product, [1] error bits,
                                    // [2..3] outputs listed since the last profile read (u64)
  int* h_oz_err = nullptr;          // pinned
  // precision
  int precision = KC_PRECISION_CERTIFIED;
  // the certification margin: kappa0 (kc_set_precision may set it) times
  // kappa_mul, which the audit of recomputed frames raises after a violation
  float kappa0 = kc::kCertKappa0, kappa_mul = 1.0f;
  float* d_audit = nullptr;         // [1] largest |s^ - s| / B over the last batch's recomputed pairs (float bits)
  float* h_audit = nullptr;         // pinned copy
  bool audit_pending = false;       // h_audit holds an unread audit
  double host_wait_ms = 0;          // time the host spent blocked in wait_stream (the stream's worker reports it)
  std::vector<void*> retired;       // workspace buffers replaced since the last stream wait (ensure)
  int sa = 10;                      // activations are split at x * 2^sa
  // test hook (kc_inject_wait_expiry): the next launch of this tensor-core
  // kernel (KC_INJECT_*) reports an expired wait before it issues any copy
  int inject = -1;
  std::vector<Mat> mats;
  std::vector<float> mat_max;       // max |W| per matrix (host side, from the last sync)
  std::vector<uint64_t> img_off;    // byte offset of each matrix's image
  // the bank-side projections that share an input, as the matrices of one
  // planes product (their images contiguous, in this order): bk through the
  // selector's Wk then each mixer block's Wk, bv through each block's Wv
  std::vector<int> kplanes, vplanes;
  DevBuf images;
  std::vector<char> mat_dirty;      // per matrix: its image is stale
  int* d_err = nullptr;             // tensor-core pipeline error word
  int* h_err = nullptr;             // pinned
  uint32_t* h_flags_pinned = nullptr;  // certify's readback (flags, per-frame t, q, r) and its frame list
  size_t h_flags_cap = 0;
  // profiling
  bool profiling = false;
  kc_stage_times prof{};
  std::vector<std::pair<cudaEvent_t, cudaEvent_t>> ev_pool;
  std::vector<std::pair<int, size_t>> ev_used;  // (stage, index into ev_pool)
  std::vector<double> ev_flops;
  std::vector<double> ev_bytes;
};

namespace {

// A workspace buffer of at least `bytes`. A buffer that must grow again gets
// an eighth more than asked, so that batches of slowly rising size (rolling
// stream batches, the varying number of recomputed frames) do not reallocate
// at every new high. The buffer it replaces may still be read by work queued
// on the stream, and cudaFree would wait for the whole device in the middle
// of a batch: it is retired instead and freed after the next stream wait.
cudaError_t ensure(kc_handle* h, DevBuf& b, size_t bytes) {
  if (bytes <= b.cap && b.p) return cudaSuccess;
  const double t0 = now_ms();
  const bool regrow = b.p != nullptr;
  if (b.p) h->retired.push_back(b.p);
  b.p = nullptr;
  b.cap = 0;
  size_t want = bytes < 256 ? 256 : bytes;
  if (regrow) want += want / 8;
  want = (want + 255) & ~size_t(255);
  cudaError_t e = cudaMalloc(&b.p, want);
  if (e == cudaSuccess) b.cap = want;
  t_grows++;
  t_grow_ms += now_ms() - t0;
  return e;
}

// Frees the buffers ensure retired; only after a wait for the stream, when
// nothing queued can still read them.
void release_retired(kc_handle* h) {
  for (void* p : h->retired) cudaFree(p);
  h->retired.clear();
}

kc_status fail(kc_handle* h, kc_status s, const std::string& msg) {
  if (h) h->err = msg;
  else g_create_error = msg;
  return s;
}

kc_status cuda_fail(kc_handle* h, cudaError_t e, const char* what) {
  return fail(h, e == cudaErrorMemoryAllocation ? KC_ERR_CAPACITY : KC_ERR_CUDA,
              std::string(what) + ": " + cudaGetErrorString(e));
}

// The batch path's host waits for its stream, timed.
cudaError_t wait_stream(kc_handle* h) {
  const double t0 = now_ms();
  const cudaError_t e = cudaStreamSynchronize(h->stream);
  h->host_wait_ms += now_ms() - t0;
  if (e == cudaSuccess && !h->retired.empty()) release_retired(h);
  return e;
}

#define KC_TRY(expr, what)                                     \
  do {                                                         \
    cudaError_t _e = (expr);                                   \
    if (_e != cudaSuccess) return cuda_fail(h, _e, what);      \
  } while (0)

#define KC_CHECK(expr)             \
  do {                             \
    kc_status _s = (expr);         \
    if (_s != KC_OK) return _s;    \
  } while (0)

// Profiling: a pair of events around each launch group.
struct ProfScope {
  kc_handle* h;
  int stage;
  size_t idx = 0;
  bool on;
  ProfScope(kc_handle* hh, int st, double flops = 0, double bytes = 0) : h(hh), stage(st), on(hh->profiling) {
    if (!on) return;
    idx = h->ev_used.size();
    if (idx >= h->ev_pool.size()) {
      cudaEvent_t a, b;
      cudaEventCreate(&a);
      cudaEventCreate(&b);
      h->ev_pool.emplace_back(a, b);
    }
    h->ev_used.emplace_back(stage, idx);
    h->ev_flops.push_back(flops);
    h->ev_bytes.push_back(bytes);
    cudaEventRecord(h->ev_pool[idx].first, h->stream);
  }
  ~ProfScope() {
    if (on) cudaEventRecord(h->ev_pool[idx].second, h->stream);
  }
};

void prof_collect(kc_handle* h) {
  if (!h->profiling || h->ev_used.empty()) return;
  cudaStreamSynchronize(h->stream);
  double* dst[kStCount] = {&h->prof.pack_ms, &h->prof.embed_ms, &h->prof.enc_gemm_ms, &h->prof.enc_attn_ms,
                           &h->prof.pool_ms, &h->prof.mixer_ms, &h->prof.selector_ms, &h->prof.fallback_ms,
                           &h->prof.enc_ffn_ms, &h->prof.enc_attn_tc_ms};
  for (size_t i = 0; i < h->ev_used.size(); i++) {
    float ms = 0;
    auto& pr = h->ev_pool[h->ev_used[i].second];
    cudaEventElapsedTime(&ms, pr.first, pr.second);
    *dst[h->ev_used[i].first] += ms;
    h->prof.total_ms += ms;
    if (h->ev_used[i].first == kStEncGemm) {
      h->prof.enc_gemm_launches++;
      h->prof.enc_gemm_flops += h->ev_flops[i];
      h->prof.enc_gemm_bytes += h->ev_bytes[i];
    } else if (h->ev_used[i].first == kStEncFfn) {
      h->prof.enc_ffn_launches++;
      h->prof.enc_ffn_flops += h->ev_flops[i];
      h->prof.enc_ffn_bytes += h->ev_bytes[i];
    } else if (h->ev_used[i].first == kStEncAttnTc) {
      h->prof.enc_attn_tc_launches++;
      h->prof.enc_attn_tc_flops += h->ev_flops[i];
      h->prof.enc_attn_tc_bytes += h->ev_bytes[i];
    }
  }
  h->ev_used.clear();
  h->ev_flops.clear();
  h->ev_bytes.clear();
}

// The exact GEMM with the largest CTA tile that still keeps most SMs busy
// (128 once its grid covers half of them: the token-parallel products; 64
// or 32 for the few rows of the recomputed frames' mixer and selector).
template <int EPI>
void launch_dgemm(kc_handle* h, const float* A, uint32_t lda, const float* B, uint32_t ldb, float* C, uint64_t M,
                  uint32_t N, uint32_t K, const float* gate) {
  const uint64_t sms = uint64_t(h->sms);
  if (2 * ((M + 127) / 128) * (N / 128) >= sms)
    kc::k_dgemm_exact<EPI, 128><<<dim3(unsigned((M + 127) / 128), N / 128), 256, 0, h->stream>>>(
        A, B, C, int(M), int(N), int(K), int(lda), int(ldb), int(N), gate);
  else if (((M + 63) / 64) * (N / 64) >= sms)
    kc::k_dgemm_exact<EPI, 64><<<dim3(unsigned((M + 63) / 64), N / 64), 256, 0, h->stream>>>(
        A, B, C, int(M), int(N), int(K), int(lda), int(ldb), int(N), gate);
  else
    kc::k_dgemm_exact<EPI, 32><<<dim3(unsigned((M + 31) / 32), N / 32), 256, 0, h->stream>>>(
        A, B, C, int(M), int(N), int(K), int(lda), int(ldb), int(N), gate);
  h->launches++;
}

template <int EPI>
kc_status dgemm(kc_handle* h, const float* A, const float* B, float* C, uint64_t M, uint32_t N, uint32_t K) {
  if (M == 0) return KC_OK;
  launch_dgemm<EPI>(h, A, K, B, K, C, M, N, K, nullptr);
  return KC_OK;
}

// As dgemm, with A's row stride and the gate of kEpiGate.
template <int EPI>
kc_status dgemm_ld(kc_handle* h, const float* A, uint32_t lda, const float* B, float* C, uint64_t M, uint32_t N,
                   uint32_t K, const float* gate = nullptr, uint32_t ldb = 0) {
  if (M == 0) return KC_OK;
  launch_dgemm<EPI>(h, A, lda, B, ldb ? ldb : K, C, M, N, K, gate);
  return KC_OK;
}

// Transposed copies of every block and selector matrix, at their page offsets
// in h->wt (the backward's input products multiply by them).
kc_status build_transposes(kc_handle* h) {
  if (!h->wt_blocks_dirty && !h->wt_sel_dirty) return KC_OK;
  const Dims& d = h->d;
  KC_TRY(ensure(h, h->wt, d.total * 4), "transposed weights");
  float* wt = P<float>(h->wt);
  auto tr = [&](uint64_t off, uint32_t n, uint32_t k) {
    dim3 grid((k + 31) / 32, (n + 31) / 32);
    kc::k_transpose<<<grid, dim3(32, 8), 0, h->stream>>>(h->w + off, wt + off, int(n), int(k));
    h->launches++;
  };
  const uint64_t hh = uint64_t(d.h) * d.h, fh = uint64_t(d.ffn) * d.h;
  for (int pass = 0; pass < 2 && h->wt_blocks_dirty; pass++) {
    const uint64_t base = pass ? d.off_mixer : d.off_enc;
    for (uint32_t b = 0; b < (pass ? d.mix : d.enc); b++) {
      const uint64_t o = base + d.block * b;
      if (pass == 0) {
        tr(o, 3 * d.h, d.h);  // [Wq; Wk; Wv] -> [Wqᵀ | Wkᵀ | Wvᵀ]
      } else {
        tr(o, d.h, d.h);
        tr(o + hh, d.h, d.h);
        tr(o + 2 * hh, d.h, d.h);
      }
      tr(o + 3 * hh, d.ffn, d.h);
      tr(o + 3 * hh + fh, d.h, d.ffn);
    }
  }
  if (h->wt_sel_dirty) {
    tr(d.off_swq, d.h, d.h);
    tr(d.off_swk, d.h, d.h);
  }
  KC_TRY(cudaGetLastError(), "transposed weights");
  h->wt_blocks_dirty = h->wt_sel_dirty = false;
  return KC_OK;
}

// Rebuild the split fp16 images of the matrices a sync changed.
kc_status build_images(kc_handle* h) {
  bool any = false;
  for (char c : h->mat_dirty) any |= c != 0;
  if (!any) return KC_OK;
  KC_CHECK(build_transposes(h));
  const auto& m = h->mats;
  if (h->img_off.size() != m.size()) {
    h->img_off.assign(m.size(), ~uint64_t(0));
    uint64_t off = 0;
    auto place = [&](int i) {
      if (h->img_off[i] != ~uint64_t(0)) return;
      h->img_off[i] = off;
      off += uint64_t(m[i].n) * m[i].k * 4;  // hi + lo fp16
    };
    for (int i : h->kplanes) place(i);  // each planes group contiguous, in plane order
    for (int i : h->vplanes) place(i);
    for (size_t i = 0; i < m.size(); i++) place(int(i));
    KC_TRY(ensure(h, h->images, off), "weight images");
  }
  for (size_t i = 0; i < m.size(); i++) {
    if (!h->mat_dirty[i]) continue;
    h->mat_dirty[i] = 0;
    const int sw = int(std::floor(std::log2(2048.0 / std::max(double(h->mat_max[i]), 1e-30))));
    const int swc = std::min(std::max(sw, -40), 40);
    const float* src = (m[i].transposed ? P<float>(h->wt) : h->w) + m[i].page_off;
    kc::tc::k_weight_image<<<(m[i].n / 128) * (m[i].k / 64), 256, 0, h->stream>>>(
        src, int(m[i].n), int(m[i].k), std::ldexp(1.0f, swc), P<uint8_t>(h->images) + h->img_off[i]);
    h->launches++;
  }
  KC_TRY(cudaGetLastError(), "weight images");
  return KC_OK;
}

int mat_sw(kc_handle* h, int i) {
  const int sw = int(std::floor(std::log2(2048.0 / std::max(double(h->mat_max[i]), 1e-30))));
  return std::min(std::max(sw, -40), 40);
}

// 1 when the test hook is armed for this kernel (and disarms it).
int take_injection(kc_handle* h, int kernel) {
  if (h->inject != kernel) return 0;
  h->inject = -1;
  return 1;
}

// The planes groups of a geometry: the selector's Wk and each mixer block's
// Wk (all read bk), each block's Wv (all read bv); empty when a group does
// not fit one planes product (square H = 128 matrices, at most kMaxPlanes).
void plan_planes(kc_handle* h) {
  const Dims& d = h->d;
  h->kplanes.clear();
  h->vplanes.clear();
  const int mix_m = 3 * int(d.enc), sel_m = mix_m + 5 * int(d.mix);
  if (d.h != 128 || d.mix == 0 || int(d.mix) + 1 > kc::tc::kMaxPlanes) return;
  h->kplanes.push_back(sel_m + 1);
  for (uint32_t b = 0; b < d.mix; b++) h->kplanes.push_back(mix_m + 5 * int(b) + 1);
  for (uint32_t b = 0; b < d.mix; b++) h->vplanes.push_back(mix_m + 5 * int(b) + 2);
}

// y = A·Wᵀ on the tensor cores for matrix `mat` of mat_list.
template <int EPI>
kc_status tc_gemm(kc_handle* h, const float* A, uint64_t M, int mat, float* C, const float* gate = nullptr) {
  if (M == 0) return KC_OK;
  const Mat& mt = h->mats[mat];
  CUtensorMap map, cmap, gmap;
  if (!kc::tc::make_a_map(&map, A, M, mt.k, mt.k) || !kc::tc::make_c_map(&cmap, C, M, mt.n, mt.n) ||
      !kc::tc::make_c_map(&gmap, gate ? gate : C, M, mt.n, mt.n))
    return fail(h, KC_ERR_CUDA, "the driver refused a tensor map for a GEMM operand");
  kc::tc::GemmArgs g{int(M), int(mt.k), int(mt.n / 128), P<uint8_t>(h->images) + h->img_off[mat], C,
                     int(mt.n), std::ldexp(1.0f, h->sa), std::ldexp(1.0f, -(h->sa + mat_sw(h, mat))), h->d_err,
                     take_injection(h, KC_INJECT_GEMM)};
  const uint64_t tiles = ((M + 127) / 128) * (mt.n / 128);
  const unsigned grid = unsigned(tiles < uint64_t(h->sms) ? tiles : uint64_t(h->sms));
  kc::tc::k_tc_gemm<EPI><<<grid, kc::tc::kThreadsT, kc::tc::kSmemBytesT, h->stream>>>(map, cmap, gmap, g);
  h->launches++;
  return KC_OK;
}

// C[p] = A·W_pᵀ for the matrices of a planes group (contiguous images, H x
// H each) in one product: A is read once for all of them, and plane p of C
// ([planes, M, 128]) holds what tc_gemm<kEpiStore> of matrix p would store.
kc_status tc_gemm_planes(kc_handle* h, const float* A, uint64_t M, const std::vector<int>& mats, float* C) {
  if (M == 0) return KC_OK;
  CUtensorMap map, cmap;
  if (!kc::tc::make_a_map(&map, A, M, 128, 128) || !kc::tc::make_c_map3(&cmap, C, M, mats.size()))
    return fail(h, KC_ERR_CUDA, "the driver refused a tensor map for a GEMM operand");
  kc::tc::GemmArgs g{int(M), 128, int(mats.size()), P<uint8_t>(h->images) + h->img_off[mats[0]], C, 128,
                     std::ldexp(1.0f, h->sa), 1.0f, h->d_err, take_injection(h, KC_INJECT_GEMM)};
  g.planes = int(mats.size());
  for (size_t p = 0; p < mats.size(); p++) g.unscale_n[p] = std::ldexp(1.0f, -(h->sa + mat_sw(h, mats[p])));
  const uint64_t tiles = ((M + 127) / 128) * mats.size();
  const unsigned grid = unsigned(tiles < uint64_t(h->sms) ? tiles : uint64_t(h->sms));
  kc::tc::k_tc_gemm<kc::tc::kEpiStore><<<grid, kc::tc::kThreadsT, kc::tc::kSmemBytesT, h->stream>>>(map, cmap, cmap, g);
  h->launches++;
  return KC_OK;
}

// x += relu(x·W1ᵀ)·W2ᵀ on the tensor cores in one kernel (ffn.cuh), for the
// W1 / W2 matrices mat_w1 / mat_w2 of the tensor-core list. Needs H = 128 and
// F = 384 (the kernel's fixed tiling); ffn_fusable() says whether it applies.
bool ffn_fusable(const kc_handle* h) { return h->fuse && h->d.h == 128 && h->d.ffn == 384; }

kc_status tc_ffn(kc_handle* h, float* x, uint64_t M, int mat_w1, int mat_w2) {
  if (M == 0) return KC_OK;
  CUtensorMap amap, cmap;
  if (!kc::tc::make_a_map(&amap, x, M, 128, 128) || !kc::tc::make_c_map(&cmap, x, M, 128, 128))
    return fail(h, KC_ERR_CUDA, "the driver refused a tensor map for the feed-forward operand");
  kc::tc::FfnArgs fa{int(M), P<uint8_t>(h->images) + h->img_off[mat_w1], P<uint8_t>(h->images) + h->img_off[mat_w2],
                     std::ldexp(1.0f, h->sa), std::ldexp(1.0f, -(h->sa + mat_sw(h, mat_w1))),
                     std::ldexp(1.0f, -(h->sa + mat_sw(h, mat_w2))), h->d_err,
                     take_injection(h, KC_INJECT_FFN)};
  const uint64_t tiles = (M + 127) / 128;
  const unsigned grid = unsigned(tiles < uint64_t(h->sms) ? tiles : uint64_t(h->sms));
  kc::tc::k_tc_ffn<<<grid, kc::tc::kThreadsT, kc::tc::kFfnSmem, h->stream>>>(amap, cmap, fa);
  h->launches++;
  return KC_OK;
}

// The per-frame cross attention's key block for a batch whose largest bank
// is max_r rows (a multiple of 32, at most kCaBlock), the length of a score
// row's parity half (16 mod 32, at least half the block), and its shared
// memory (the k block buffer, the scores, the question rows).
struct CrossShape {
  int kb, half;
  size_t smem;
};
CrossShape cross_shape(uint32_t max_r) {
  const int kb = int(std::min<uint32_t>(kc::kCaBlock, (std::max<uint32_t>(max_r, 1) + 31) / 32 * 32));
  const int half = (kb / 2 + 31) / 32 * 32 + 16;
  return {kb, half,
          size_t(kc::kCaBlock) * KC_H * 4 + size_t(kc::kCaChunk) * KC_HEADS * 2 * half * 4 +
              size_t(kc::kCaChunk) * KC_H * 4};
}

// The one-pass cross attention's score-row parity half for banks of at most
// max_r rows (16 mod 32, at least half the longest bank) and its shared memory
// (scores [kCsChunk][4][2*half], q [kCsChunk][128], then a block of kCsKeys
// k rows).
int cross_small_half(uint32_t max_r) {
  return int((std::max<uint32_t>(max_r, 1) + 1) / 2 + 31) / 32 * 32 + 16;
}
size_t cross_small_smem(uint32_t max_r) {
  return size_t(kc::kCsChunk) * KC_HEADS * 2 * cross_small_half(max_r) * 4 + size_t(kc::kCsChunk) * KC_H * 4 +
         size_t(kc::kCsKeys) * KC_H * 4;
}

// The same for the per-frame selector (scores [qc][max_r], then q [qc][128]).
int sel_chunk(uint32_t max_r) {
  const uint64_t fit = (96u << 10) / (4ull * std::max<uint32_t>(max_r, 1));
  return int(std::min<uint64_t>(std::max<uint64_t>(fit, 1), kc::kSelChunk));
}
size_t sel_smem(uint32_t max_r) {
  const int qc = sel_chunk(max_r);
  return size_t(qc) * std::max<uint32_t>(max_r, 1) * 4 + size_t(qc) * KC_H * 4;
}

// qkv = x·Wqkvᵀ, record-local attention and x += o in one kernel
// (attn_tc.cuh) for the encoder block whose Wqkv is `mat`. Needs H = 128 and
// a head dim of 32 (the kernel's fixed tiling); attn_fusable() says whether it
// applies.
bool attn_fusable(const kc_handle* h) { return h->fuse && h->d.h == 128 && h->d.hd == 32 && h->d.heads == 4; }

uint64_t attn_tiles(uint64_t T) { return (T + kc::tc::kAtWindow - 1) / kc::tc::kAtWindow; }

// The tile table and row info of a packed batch (once per batch).
kc_status attn_prepare(kc_handle* h, Workspace& ws, uint64_t T) {
  if (T == 0) return KC_OK;
  const uint64_t tiles = attn_tiles(T);
  KC_TRY(ensure(h, ws.tile_row, (tiles + 1) * 4), "workspace");
  KC_TRY(ensure(h, ws.row_rc, T * 4), "workspace");
  kc::tc::k_attn_tiles<<<unsigned((T + 255) / 256), 256, 0, h->stream>>>(
      P<uint32_t>(ws.tok_recpos), P<uint32_t>(ws.rec_start), P<uint2>(ws.rec_meta), int(T), int(tiles),
      P<uint32_t>(ws.row_rc), P<int>(ws.tile_row));
  h->launches++;
  return KC_OK;
}

kc_status tc_attn(kc_handle* h, Workspace& ws, float* x, uint64_t T, int mat, const uint32_t* word_ids,
                  float word_alpha, float scale) {
  if (T == 0) return KC_OK;
  CUtensorMap xmap;
  if (!kc::tc::make_x_map(&xmap, x, T))
    return fail(h, KC_ERR_CUDA, "the driver refused a tensor map for the attention operand");
  kc::tc::AttnTcArgs aa{};
  aa.T = int(T);
  aa.tiles = int(attn_tiles(T));
  aa.tile_row = P<int>(ws.tile_row);
  aa.row_rc = P<uint32_t>(ws.row_rc);
  aa.w = P<uint8_t>(h->images) + h->img_off[mat];
  aa.a_scale = std::ldexp(1.0f, h->sa);
  aa.unscale = std::ldexp(1.0f, -(h->sa + mat_sw(h, mat)));
  aa.x = x; aa.tok_recpos = P<uint32_t>(ws.tok_recpos);
  aa.word_ids = word_alpha != 0.0f ? word_ids : nullptr;
  aa.word_alpha = word_alpha; aa.scale = scale; aa.err = h->d_err;
  aa.inject_expiry = take_injection(h, KC_INJECT_ATTN);
  const unsigned grid = unsigned(std::min<uint64_t>(uint64_t(aa.tiles), uint64_t(h->sms)));
  if (aa.word_ids)
    kc::tc::k_tc_attn<true><<<grid, kc::tc::kAtThreads, kc::tc::kAtSmem, h->stream>>>(xmap, aa);
  else
    kc::tc::k_tc_attn<false><<<grid, kc::tc::kAtThreads, kc::tc::kAtSmem, h->stream>>>(xmap, aa);
  h->launches++;
  return KC_OK;
}

// Whether an exact-path product runs on the int8 tensor cores: a forward
// matrix of the list read from the weight page, K a multiple of 128 up to
// 384, N a multiple of 64, A, C and the gate 16-byte aligned, and enough rows
// to fill the GPU (a few dozen recomputed frames' question or bank rows take
// one FP64 launch instead of the slicing, product and fixup launches).
constexpr uint64_t kOzMinRows = 16384;
bool oz_fits(const kc_handle* h, const float* A, uint32_t lda, uint64_t M, int mat, const float* B, uint32_t ldb,
             float* C, const float* gate, uint32_t N, uint32_t K) {
  if (M < kOzMinRows) return false;
  const auto aligned = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (!aligned(C) || (gate && !aligned(gate))) return false;
  if (!h->oz || h->oz_suspend || mat < 0 || size_t(mat) >= h->mats.size()) return false;
  const Mat& mt = h->mats[mat];
  return !mt.transposed && mt.page_off % 4 == 0 && mt.n == N && mt.k == K && B == h->w + mt.page_off && ldb == K &&
         K % 128 == 0 &&
         K <= uint32_t(kc::oz::kMaxK) && N % 64 == 0 && lda % 4 == 0 && (reinterpret_cast<uintptr_t>(A) & 15) == 0;
}

// The slices and row data of forward matrix `mat` (rebuilt after a sync
// changed it): [6][N][K] int8, then l1, l2, the column scale 2^e and the
// bound's column term [N] (f64), e [N] (int).
kc_status oz_weights(kc_handle* h, int mat) {
  const auto& m = h->mats;
  if (h->oz_w_off.size() != m.size()) {
    h->oz_w_off.assign(m.size(), 0);
    uint64_t off = 0;
    for (size_t i = 0; i < m.size(); i++) {
      if (m[i].transposed) continue;
      h->oz_w_off[i] = off;
      off += (uint64_t(m[i].n) * m[i].k * kc::oz::kSlices + uint64_t(m[i].n) * 36 + 255) & ~uint64_t(255);
    }
    KC_TRY(ensure(h, h->oz_w, off), "weight slices");
  }
  if (!h->oz_dirty[mat]) return KC_OK;
  h->oz_dirty[mat] = 0;
  const Mat& mt = m[mat];
  uint8_t* base = P<uint8_t>(h->oz_w) + h->oz_w_off[mat];
  const uint64_t plane = uint64_t(mt.n) * mt.k;
  double* l1 = reinterpret_cast<double*>(base + plane * kc::oz::kSlices);
  kc::oz::SliceArgs sa{h->w + mt.page_off, mt.n, int(mt.k), mt.k, base, plane, reinterpret_cast<int*>(l1 + 4 * mt.n),
                       l1, l1 + mt.n, nullptr};
  sa.col_s = l1 + 2 * mt.n;
  sa.col_p = l1 + 3 * mt.n;
  sa.c2k = std::ldexp(double(mt.k), -94) + kc::oz::dropped_levels_bound(int(mt.k));
  kc::oz::k_oz_slice<<<(mt.n + 7) / 8, 256, 0, h->stream>>>(sa);
  h->launches++;
  KC_TRY(cudaGetLastError(), "weight slices");
  return KC_OK;
}

// C (= epilogue) A·Wᵀ for forward matrix `mat` on the int8 tensor cores:
// slice A, the product (outputs it cannot settle are listed), the listed
// outputs by the sequential chain. The same f32 results as dgemm.
template <int EPI>
kc_status oz_gemm(kc_handle* h, const float* A, uint32_t lda, uint64_t M, int mat, float* C, uint32_t N, uint32_t K,
                  const float* gate) {
  if (M == 0) return KC_OK;
  KC_CHECK(oz_weights(h, mat));
  const Mat& mt = h->mats[mat];
  const uint64_t plane = M * K;
  KC_TRY(ensure(h, h->oz_a, plane * kc::oz::kSlices), "workspace");
  KC_TRY(ensure(h, h->oz_meta, M * 20), "workspace");
  const uint64_t cap = h->oz_cap >= 0 ? uint64_t(h->oz_cap) : std::max<uint64_t>(65536, M * N / 128);
  KC_TRY(ensure(h, h->oz_list, cap * 8), "workspace");
  double* l1a = P<double>(h->oz_meta);
  int* ea = reinterpret_cast<int*>(l1a + 2 * M);
  unsigned* count = h->d_oz_word;
  kc::oz::SliceArgs sa{A, M, int(K), lda, P<uint8_t>(h->oz_a), plane, ea, l1a, l1a + M, count};
  kc::oz::k_oz_slice<<<unsigned((M + 7) / 8), 256, 0, h->stream>>>(sa);
  const uint8_t* wb = P<uint8_t>(h->oz_w) + h->oz_w_off[mat];
  const uint64_t wplane = uint64_t(mt.n) * mt.k;
  const double* l1b = reinterpret_cast<const double*>(wb + wplane * kc::oz::kSlices);
  CUtensorMap amap, bmap;
  if (!kc::oz::make_slice_map(&amap, P<uint8_t>(h->oz_a), M, K, kc::oz::kBM) ||
      !kc::oz::make_slice_map(&bmap, wb, N, K, kc::oz::kBN))
    return fail(h, KC_ERR_CUDA, "the driver refused a tensor map for a sliced operand");
  kc::oz::GemmArgs g{};
  g.M = int(M); g.N = int(N); g.K = int(K);
  g.ea = ea; g.l1a = l1a; g.l2a = l1a + M;
  g.sb = l1b + 2 * mt.n; g.pb = l1b + 3 * mt.n; g.l2b = l1b + mt.n;
  g.C = C; g.ldc = int(N); g.gate = gate;
  g.list = P<unsigned long long>(h->oz_list); g.count = count; g.cap = unsigned(cap);
  g.err = reinterpret_cast<int*>(count + 1);
  g.gamma = kc::oz::chain_gamma(int(K));
  g.inject_expiry = take_injection(h, KC_INJECT_EXACT_GEMM);
  const uint64_t tiles = ((M + kc::oz::kBM - 1) / kc::oz::kBM) * (N / kc::oz::kBN);
  const unsigned grid = unsigned(std::min<uint64_t>(tiles, uint64_t(h->sms)));
  kc::oz::k_oz_gemm<EPI><<<grid, kc::oz::kThreads, kc::oz::kSmem, h->stream>>>(amap, bmap, g);
  kc::oz::FixupArgs fx{A, lda, h->w + mt.page_off, K, int(K), C, int(N), gate, g.list, count, unsigned(cap),
                       reinterpret_cast<unsigned long long*>(count + 2)};
  kc::oz::k_oz_fixup<EPI><<<unsigned(h->sms) * 2, 256, 0, h->stream>>>(fx);
  h->launches += 3;
  h->oz_ran = true;
  h->prof.oz_products++;
  h->prof.oz_outputs += double(M) * N;
  KC_TRY(cudaGetLastError(), "sliced product");
  return KC_OK;
}

// One GEMM of the exact sequence: on the FP64 pipe in the oracle's order (or
// with the same results on the int8 tensor cores, oz_gemm), or (tc) on the
// split-fp16 tensor cores, where `mat` names the matrix in the tensor-core
// list and B / ldb the same matrix for the FP64 kernel. The tensor-core path
// reads A with row stride K.
template <int EPI>
kc_status gemm(kc_handle* h, bool tc, const float* A, uint32_t lda, uint64_t M, int mat, const float* B,
               uint32_t ldb, float* C, uint32_t N, uint32_t K, const float* gate = nullptr) {
  if (tc) return tc_gemm<EPI>(h, A, M, mat, C, gate);
  if (oz_fits(h, A, lda, M, mat, B, ldb, C, gate, N, K)) return oz_gemm<EPI>(h, A, lda, M, mat, C, N, K, gate);
  return dgemm_ld<EPI>(h, A, lda, B, C, M, N, K, gate, ldb);
}

// Device-side view of one batch (all pointers on the handle's device).
struct DevBatch {
  uint32_t frames = 0;
  uint64_t records = 0;
  const uint64_t* rec_off = nullptr;
  const uint32_t *token_ids = nullptr, *field_roles = nullptr, *schema_ids = nullptr, *band_ids = nullptr;
  const uint32_t *schema_allow = nullptr, *band_allow = nullptr;
  const double* uniforms = nullptr;
  const uint32_t* word_ids = nullptr;  // the same-word bias (null or alpha 0: none)
  float word_alpha = 0.0f;
  const float* mask = nullptr;         // explicit selection mask laid out like p (null: the rule, or open)
  uint64_t mask_len = UINT64_MAX;      // its entries when staged here (checked against the packed size)
};

const char* bad_message(uint32_t code) {
  switch (code) {
    case kc::kBadTokenId: return "token id has no entry in tokenRows";
    case kc::kBadTokenRow: return "token row outside the token table";
    case kc::kBadRoleId: return "field role id has no entry in tokenRows";
    case kc::kBadRoleRow: return "field role row outside the field table";
    case kc::kBadSchema: return "schema id outside the schema table";
    case kc::kBadBand: return "band id outside the band table";
    case kc::kBadEmptyFrame: return "a frame with no records has nothing to think about";
    case kc::kBadBank: return "bank exceeds capacity";
    default: return "malformed frame";
  }
}

// Pack on the GPU: offset tables, compact token list, row lists. One host
// wait for the batch totals (sizes the rest of the workspace), unless the
// caller knows them (`known`: a sub-batch of frames an earlier pack checked).
kc_status pack_batch(kc_handle* h, Workspace& ws, const DevBatch& b, kc::FrameTotals* out_tot,
                     const kc::FrameTotals* known = nullptr) {
  const Dims& d = h->d;
  if (&ws == &h->ws) h->ws_epoch++;
  const uint32_t F = b.frames;
  const uint64_t N = b.records;
  if (F == 0) return fail(h, KC_ERR_INVALID_ARG, "a batch with no frames");
  KC_TRY(ensure(h, ws.rec_meta, N * sizeof(uint2)), "workspace");
  KC_TRY(ensure(h, ws.frame_t, F * 4ull), "workspace");
  KC_TRY(ensure(h, ws.frame_q, F * 4ull), "workspace");
  KC_TRY(ensure(h, ws.frame_r, F * 4ull), "workspace");
  KC_TRY(ensure(h, ws.t_off, (F + 1) * 8ull), "workspace");
  KC_TRY(ensure(h, ws.q_off, (F + 1) * 8ull), "workspace");
  KC_TRY(ensure(h, ws.r_off, (F + 1) * 8ull), "workspace");
  KC_TRY(ensure(h, ws.p_off, (F + 1) * 8ull), "workspace");
  KC_TRY(ensure(h, ws.totals, sizeof(kc::FrameTotals)), "workspace");
  KC_TRY(ensure(h, ws.rec_start, N * 4), "workspace");
  KC_TRY(ensure(h, ws.rec_row, N * 4), "workspace");
  kc::FrameTotals* dtot = P<kc::FrameTotals>(ws.totals);
  {
    ProfScope ps(h, kStPack);
    KC_TRY(cudaMemsetAsync(dtot, 0, sizeof(kc::FrameTotals), h->stream), "memset");
    kc::k_frame_scan<256><<<F, 256, 0, h->stream>>>(
        b.rec_off, F, b.token_ids, b.field_roles, b.schema_ids, b.band_ids, h->token_rows, h->token_rows_len,
        d.token_space, d.field_space, d.schema_space, d.band_space, KC_MAX_BANK, P<uint2>(ws.rec_meta),
        P<uint32_t>(ws.frame_t), P<uint32_t>(ws.frame_q), P<uint32_t>(ws.frame_r), dtot);
    kc::k_frame_offsets<1024><<<1, 1024, 0, h->stream>>>(F, P<uint32_t>(ws.frame_t), P<uint32_t>(ws.frame_q),
                                                          P<uint32_t>(ws.frame_r), P<uint64_t>(ws.t_off),
                                                          P<uint64_t>(ws.q_off), P<uint64_t>(ws.r_off),
                                                          P<uint64_t>(ws.p_off), dtot);
    h->launches += 2;
    if (!known)
      KC_TRY(cudaMemcpyAsync(h->h_tot, dtot, sizeof(kc::FrameTotals), cudaMemcpyDeviceToHost, h->stream),
             "readback");
  }
  if (!known) KC_TRY(wait_stream(h), "pack");
  const kc::FrameTotals tot = known ? *known : *h->h_tot;
  if (tot.bad) {
    char buf[160];
    snprintf(buf, sizeof buf, "%s (%s %u)", bad_message(tot.bad),
             tot.bad == kc::kBadEmptyFrame || tot.bad == kc::kBadBank ? "frame" : "record", tot.bad_where);
    if (tot.bad == kc::kBadBank)
      snprintf(buf, sizeof buf, "bank records of frame %u exceed capacity %u", tot.bad_where, KC_MAX_BANK);
    return fail(h, tot.bad == kc::kBadBank ? KC_ERR_CAPACITY : KC_ERR_INVALID_ARG, buf);
  }
  const uint64_t T = tot.t, Q = tot.q, R = tot.r, PP = tot.p;
  const uint32_t H = d.h, FF = d.ffn;
  KC_TRY(ensure(h, ws.tok_recpos, T * 4), "workspace");
  KC_TRY(ensure(h, ws.bank_rec, R * 4), "workspace");
  KC_TRY(ensure(h, ws.bank_frame, R * 4), "workspace");
  KC_TRY(ensure(h, ws.query_rec, Q * 4), "workspace");
  KC_TRY(ensure(h, ws.query_frame, Q * 4), "workspace");
  KC_TRY(ensure(h, ws.x, T * H * 4), "workspace");
  KC_TRY(ensure(h, ws.qkv, T * (3 * H > FF ? 3 * H : FF) * 4ull), "workspace");
  KC_TRY(ensure(h, ws.bk, R * H * 4), "workspace");
  KC_TRY(ensure(h, ws.bv, R * H * 4), "workspace");
  KC_TRY(ensure(h, ws.mk, R * H * 4), "workspace");
  KC_TRY(ensure(h, ws.mv, R * H * 4), "workspace");
  KC_TRY(ensure(h, ws.sk, R * H * 4), "workspace");
  KC_TRY(ensure(h, ws.qstate, Q * H * 4), "workspace");
  KC_TRY(ensure(h, ws.mq, Q * H * 4), "workspace");
  KC_TRY(ensure(h, ws.sq, Q * H * 4), "workspace");
  KC_TRY(ensure(h, ws.mh, Q * FF * 4ull), "workspace");
  KC_TRY(ensure(h, ws.p, PP * 4), "workspace");
  KC_TRY(ensure(h, ws.index, Q * 4), "workspace");
  KC_TRY(ensure(h, ws.flags, F * 4ull), "workspace");
  KC_TRY(ensure(h, ws.nq, Q * 4), "workspace");
  KC_TRY(ensure(h, ws.nk, R * 4), "workspace");
  KC_TRY(ensure(h, ws.kappa, Q * 4), "workspace");
  {
    ProfScope ps(h, kStPack);
    kc::k_record_rows<256><<<F, 256, 0, h->stream>>>(
        b.rec_off, F, b.token_ids, P<uint2>(ws.rec_meta), P<uint64_t>(ws.t_off), P<uint64_t>(ws.q_off),
        P<uint64_t>(ws.r_off), P<uint32_t>(ws.tok_recpos), P<uint32_t>(ws.rec_start), P<uint32_t>(ws.rec_row),
        P<uint32_t>(ws.bank_rec), P<uint32_t>(ws.query_rec), P<uint32_t>(ws.query_frame),
        P<uint32_t>(ws.bank_frame));
    h->launches++;
  }
  *out_tot = tot;
  return KC_OK;
}

// What the backward needs from the forward, per block: the encoder's q|k|v,
// local-attention p and ReLU output; the mixer's projections, p and ReLU
// output. The selector then runs under `mask` and writes the soft gather.
struct Saves {
  float *enc_qkv, *enc_p, *enc_h1;                  // strides T*3H, T*32, T*F
  float *mix_q, *mix_k, *mix_v, *mix_p, *mix_h1;    // strides Q*H, R*H, R*H, 4*P, Q*F
  const float* mask;                                // [P]
  float* gather;                                    // [Q,H]
};

// The exact selection over the resident sq / sk of a packed batch: the rule
// and uniforms of b, or (the backward) an explicit mask, no sampling and the
// soft gather into `gather`.
// selectorOracle in the exact arithmetic: the masked scores for chunks of a
// frame's questions (k_select_scores_exact, into p), then softmax, the
// decision and the gather one question per CTA (k_select_exact).
void select_exact(kc_handle* h, const kc::SelectArgs& sa, uint32_t frames, uint32_t max_q, uint32_t q,
                  uint32_t max_r) {
  if (q == 0) return;
  const int chunks = int((std::max<uint32_t>(max_q, 1) + kc::kXsChunk - 1) / kc::kXsChunk);
  kc::k_select_scores_exact<<<frames * unsigned(chunks), kc::kXsThreads, kc::kXsSmem, h->stream>>>(sa, chunks);
  kc::k_select_exact<<<q, 256, size_t(std::max<uint32_t>(max_r, 1)) * 12, h->stream>>>(sa);
  h->launches += 2;
}

void launch_select_exact(kc_handle* h, Workspace& ws, const DevBatch& b, const kc::FrameTotals& tot,
                         const float* mask, float* gather) {
  kc::SelectArgs sa{};
  sa.sq = P<float>(ws.sq); sa.sk = P<float>(ws.sk); sa.bank_values = nullptr;
  sa.query_frame = P<uint32_t>(ws.query_frame); sa.r_off = P<uint64_t>(ws.r_off);
  sa.q_off = P<uint64_t>(ws.q_off); sa.p_off = P<uint64_t>(ws.p_off);
  sa.mask = nullptr; sa.schema_allow = b.schema_allow; sa.band_allow = b.band_allow;
  sa.bank_rec = P<uint32_t>(ws.bank_rec); sa.schema_ids = b.schema_ids; sa.band_ids = b.band_ids;
  sa.uniforms = b.uniforms; sa.max_r = tot.max_r; sa.scale = 1.0 / std::sqrt(double(h->d.h));
  sa.p = P<float>(ws.p); sa.index = P<uint32_t>(ws.index); sa.gather = nullptr;
  if (mask) {
    sa.mask = mask; sa.schema_allow = nullptr; sa.band_allow = nullptr; sa.uniforms = nullptr;
    sa.bank_values = P<float>(ws.bv); sa.gather = gather;
  } else if (b.mask) {  // a batch's explicit mask, in place of the rule
    sa.mask = b.mask; sa.schema_allow = nullptr; sa.band_allow = nullptr;
  }
  select_exact(h, sa, b.frames, tot.max_q, uint32_t(tot.q), tot.max_r);
}


// fieldEmbed for the batch's T tokens (k_embed_exact): one CTA per SM, the
// small tables staged in shared memory when they fit.
void launch_embed(kc_handle* h, Workspace& ws, const DevBatch& b, float* x, uint64_t T) {
  const Dims& d = h->d;
  const uint64_t small = d.tb_pos + uint64_t(d.pos_space) * d.h - d.tb_schema;  // floats, schema..pos
  const size_t bytes = kc::embed_smem_bytes(d.schema_space, uint64_t(d.band_space) + d.stream_space + d.pos_space);
  const bool staged = bytes <= kc::kEmbedSmemMax && (d.tb_schema & 3) == 0 && d.h == KC_H;
  const size_t smem = staged ? bytes : 0;
  kc::EmbedArgs ea{P<uint32_t>(ws.tok_recpos), b.token_ids, b.field_roles, b.schema_ids, b.band_ids,
                   h->token_rows, h->w, d.tb_token, d.tb_field, d.tb_schema, d.tb_band, d.tb_stream, d.tb_pos,
                   x, T, staged ? small : 0};
  const uint64_t groups = (T + kc::kEmbedTokensPerWarp - 1) / kc::kEmbedTokensPerWarp;
  const unsigned blocks = unsigned(std::min<uint64_t>(uint64_t(h->sms), (groups + kc::kEmbedWarps - 1) / kc::kEmbedWarps));
  kc::k_embed_exact<<<blocks, kc::kEmbedWarps * 32, smem, h->stream>>>(ea);
  h->launches++;
}

// The forward in the oracle's exact arithmetic (exact.cuh). Results stay in
// the workspace: qstate [Q,H], bk/bv [R,H], p, index.
kc_status forward_exact_pass(kc_handle* h, Workspace& ws, const DevBatch& b, const kc::FrameTotals& tot,
                             bool encode_only, const Saves* sv, bool tc) {
  const Dims& d = h->d;
  const uint64_t N = b.records, T = tot.t, Q = tot.q, R = tot.r;
  const uint32_t H = d.h, FF = d.ffn;
  float* x = P<float>(ws.x);
  float* qkv = P<float>(ws.qkv);
  if (T > 0) {
    ProfScope ps(h, kStEmbed);
    launch_embed(h, ws, b, x, T);
  }
  const double attn_scale = 1.0 / std::sqrt(double(d.hd));
  const double h_scale = 1.0 / std::sqrt(double(H));
  for (uint32_t blk = 0; blk < d.enc && T > 0; blk++) {
    const float* W = h->w + d.off_enc + d.block * blk;
    const float* w1 = W + 3ull * H * H;
    const float* w2 = w1 + uint64_t(FF) * H;
    float* bqkv = sv ? sv->enc_qkv + blk * T * 3 * H : qkv;
    float* bh1 = sv ? sv->enc_h1 + blk * T * FF : qkv;
    const int em = 3 * int(blk);  // this block's matrices in the tensor-core list
    {
      ProfScope ps(h, kStEncGemm, 2.0 * T * H * 3 * H, 4.0 * T * (H + 3 * H));
      KC_CHECK(gemm<kc::kEpiStore>(h, tc, x, H, T, em, W, H, bqkv, 3 * H, H));
    }
    if (tc) {  // the tensor-core forward (the batch backward's): f32 attention, its softmax rows saved
      ProfScope ps(h, kStEncAttn);
      kc::LocalAttnFastArgs la{bqkv, x, P<uint32_t>(ws.rec_start), P<uint2>(ws.rec_meta), N, float(attn_scale),
                               P<uint32_t>(ws.tok_recpos), b.word_alpha != 0.0f ? b.word_ids : nullptr,
                               b.word_alpha, sv ? sv->enc_p + blk * T * 32 : nullptr};
      kc::k_local_attn_fast<<<unsigned((N + kc::kLaWarps - 1) / kc::kLaWarps), kc::kLaWarps * 32, 0,
                              h->stream>>>(la);
      h->launches++;
    } else {
      ProfScope ps(h, kStEncAttn);
      kc::LocalAttnArgs la{bqkv, x, P<uint32_t>(ws.rec_start), P<uint2>(ws.rec_meta), N, attn_scale,
                           sv ? sv->enc_p + blk * T * 32 : nullptr, P<uint32_t>(ws.tok_recpos),
                           b.word_alpha != 0.0f ? b.word_ids : nullptr, b.word_alpha};
      kc::k_local_attn_exact<<<unsigned((N + 3) / 4), 128, 0, h->stream>>>(la);
      h->launches++;
    }
    {
      ProfScope ps(h, kStEncGemm, 2.0 * T * H * FF, 4.0 * T * (H + FF));
      KC_CHECK(gemm<kc::kEpiRelu>(h, tc, x, H, T, em + 1, w1, H, bh1, FF, H));
    }
    {
      ProfScope ps(h, kStEncGemm, 2.0 * T * H * FF, 4.0 * T * (FF + 2 * H));
      KC_CHECK(gemm<kc::kEpiResid>(h, tc, bh1, FF, T, em + 2, w2, FF, x, H, FF));
    }
  }
  {
    ProfScope ps(h, kStPool);
    kc::PoolArgs pa{x, h->w + d.off_pool, P<uint32_t>(ws.rec_start), P<uint2>(ws.rec_meta), P<uint32_t>(ws.rec_row),
                    N, h_scale, P<float>(ws.bk), P<float>(ws.bv), P<float>(ws.qstate)};
    kc::k_pool_exact<<<unsigned((N + 7) / 8), 256, 0, h->stream>>>(pa);
    h->launches++;
  }
  if (Q > 0) {
    ProfScope ps(h, kStMixer);
    for (uint32_t blk = 0; blk < d.mix; blk++) {
      const float* W = h->w + d.off_mixer + d.block * blk;
      const float* w1 = W + 3ull * H * H;
      const float* w2 = w1 + uint64_t(FF) * H;
      float* mq = sv ? sv->mix_q + blk * Q * H : P<float>(ws.mq);
      float* mk = sv ? sv->mix_k + blk * R * H : P<float>(ws.mk);
      float* mv = sv ? sv->mix_v + blk * R * H : P<float>(ws.mv);
      float* mh = sv ? sv->mix_h1 + blk * Q * FF : P<float>(ws.mh);
      const int m0 = 3 * int(d.enc) + 5 * int(blk);
      KC_CHECK(gemm<kc::kEpiStore>(h, tc, P<float>(ws.qstate), H, Q, m0, W, H, mq, H, H));
      KC_CHECK(gemm<kc::kEpiStore>(h, tc, P<float>(ws.bk), H, R, m0 + 1, W + uint64_t(H) * H, H, mk, H, H));
      KC_CHECK(gemm<kc::kEpiStore>(h, tc, P<float>(ws.bv), H, R, m0 + 2, W + 2ull * H * H, H, mv, H, H));
      // the smallest question chunk that holds the largest frame's questions,
      // smaller still while the grid would not fill two CTAs per SM (few
      // frames, e.g. the recomputed ones)
      const uint32_t mq1 = std::max<uint32_t>(tot.max_q, 1);
      int qc = 16;
      while (qc > 4 && uint32_t(qc / 2) >= mq1) qc /= 2;
      while (qc > 4 && uint64_t(b.frames) * ((mq1 + qc - 1) / qc) < 2ull * uint64_t(h->sms)) qc /= 2;
      const int chunks = int((mq1 + qc - 1) / qc);
      kc::CrossAttnArgs ca{mq, mk, mv, P<float>(ws.qstate), P<uint64_t>(ws.q_off), P<uint64_t>(ws.r_off),
                           chunks, attn_scale, sv ? sv->mix_p + blk * 4 * tot.p : nullptr,
                           P<uint64_t>(ws.p_off), tot.p};
      const unsigned grid = b.frames * unsigned(chunks);
      if (qc == 16) kc::k_cross_attn_exact<16><<<grid, kc::kXaThreads, kc::xa_smem(16), h->stream>>>(ca);
      else if (qc == 8) kc::k_cross_attn_exact<8><<<grid, kc::kXaThreads, kc::xa_smem(8), h->stream>>>(ca);
      else kc::k_cross_attn_exact<4><<<grid, kc::kXaThreads, kc::xa_smem(4), h->stream>>>(ca);
      h->launches++;
      KC_CHECK(gemm<kc::kEpiRelu>(h, tc, P<float>(ws.qstate), H, Q, m0 + 3, w1, H, mh, FF, H));
      KC_CHECK(gemm<kc::kEpiResid>(h, tc, mh, FF, Q, m0 + 4, w2, FF, P<float>(ws.qstate), H, FF));
    }
  }
  if (!encode_only && Q > 0) {
    ProfScope ps(h, kStSelector);
    const int sm = 3 * int(d.enc) + 5 * int(d.mix);
    KC_CHECK(gemm<kc::kEpiStore>(h, tc, P<float>(ws.qstate), H, Q, sm, h->w + d.off_swq, H, P<float>(ws.sq), H, H));
    KC_CHECK(gemm<kc::kEpiStore>(h, tc, P<float>(ws.bk), H, R, sm + 1, h->w + d.off_swk, H, P<float>(ws.sk), H, H));
    launch_select_exact(h, ws, b, tot, sv ? sv->mask : nullptr, sv ? sv->gather : nullptr);
  }
  KC_TRY(cudaGetLastError(), "launch");
  return KC_OK;
}

// forward_exact_pass, whose products run on the int8 tensor cores where they
// fit (oz_gemm). Their error word is read once at the end: an expired wait
// fails the call; a product that listed more outputs than its list holds
// sends the whole forward again through the FP64 kernel.
kc_status forward_exact(kc_handle* h, Workspace& ws, const DevBatch& b, const kc::FrameTotals& tot,
                        bool encode_only, const Saves* sv = nullptr, bool tc = false) {
  const bool armed = !tc && h->oz && !h->oz_suspend;
  if (armed) {
    h->oz_ran = false;
    KC_TRY(cudaMemsetAsync(h->d_oz_word + 1, 0, sizeof(unsigned), h->stream), "memset");
  }
  kc_status s = forward_exact_pass(h, ws, b, tot, encode_only, sv, tc);
  if (s || !armed || !h->oz_ran) return s;
  KC_TRY(cudaMemcpyAsync(h->h_oz_err, h->d_oz_word + 1, sizeof(int), cudaMemcpyDeviceToHost, h->stream),
         "readback");
  KC_TRY(wait_stream(h), "exact");
  const int e = *h->h_oz_err;
  if (e & kc::tc::kErrTimeout)
    return fail(h, KC_ERR_TIMEOUT, "a tensor-core pipeline wait expired; the batch was not completed");
  if (e & kc::oz::kOzListFull) {
    h->prof.oz_reruns++;
    h->oz_suspend = true;
    s = forward_exact_pass(h, ws, b, tot, encode_only, sv, tc);
    h->oz_suspend = false;
  }
  return s;
}

// The certified selection over the resident sq / sk of a packed batch: p,
// indices and the per-frame flags of decisions it cannot certify.
void launch_select_fast(kc_handle* h, Workspace& ws, const DevBatch& b, const kc::FrameTotals& tot) {
  kc::SelectFastArgs sa{};
  sa.sq = P<float>(ws.sq); sa.sk = P<float>(ws.sk);
  sa.r_off = P<uint64_t>(ws.r_off);
  sa.q_off = P<uint64_t>(ws.q_off); sa.p_off = P<uint64_t>(ws.p_off);
  sa.schema_allow = b.schema_allow; sa.band_allow = b.band_allow;
  sa.bank_rec = P<uint32_t>(ws.bank_rec); sa.schema_ids = b.schema_ids; sa.band_ids = b.band_ids;
  sa.mask = b.mask;
  if (b.mask) sa.schema_allow = sa.band_allow = nullptr;
  sa.uniforms = b.uniforms; sa.max_r = std::max<uint32_t>(tot.max_r, 1); sa.qc = sel_chunk(tot.max_r);
  sa.chunks = int((std::max<uint32_t>(tot.max_q, 1) + sa.qc - 1) / sa.qc);
  sa.scale = float(1.0 / std::sqrt(double(h->d.h)));
  sa.nq = P<float>(ws.nq); sa.nk = P<float>(ws.nk); sa.kappa = P<float>(ws.kappa);
  sa.kappa0 = h->kappa0 * h->kappa_mul; sa.lam0 = kc::kCertLam0;
  sa.p = P<float>(ws.p); sa.index = P<uint32_t>(ws.index); sa.flags = P<uint32_t>(ws.flags);
  if (tot.q) {
    kc::k_row_norms<<<unsigned((tot.q + 7) / 8), 256, 0, h->stream>>>(sa.sq, tot.q, P<float>(ws.nq));
    h->launches++;
  }
  if (tot.r) {
    kc::k_row_norms<<<unsigned((tot.r + 7) / 8), 256, 0, h->stream>>>(sa.sk, tot.r, P<float>(ws.nk));
    h->launches++;
  }
  sa.scores_in_p = tot.max_r > uint32_t(kc::kCsMaxBank);
  if (sa.scores_in_p) {  // long banks: the dot products for 16-question chunks, the bank read once per chunk
    const int chunks = int((std::max<uint32_t>(tot.max_q, 1) + kc::kSsChunk - 1) / kc::kSsChunk);
    kc::k_select_scores_fast<<<b.frames * unsigned(chunks), kc::kSsThreads, kc::kSsSmem, h->stream>>>(sa, chunks);
    h->launches++;
  }
  kc::k_select_fast<<<b.frames * unsigned(sa.chunks), 256, sel_smem(tot.max_r), h->stream>>>(sa);
  h->launches++;
}

// The forward on the tensor cores (tc_gemm.cuh, fast.cuh): the selector
// raises ws.flags[f] for frames whose decisions it cannot certify.
kc_status forward_fast(kc_handle* h, Workspace& ws, const DevBatch& b, const kc::FrameTotals& tot) {
  const Dims& d = h->d;
  const uint64_t N = b.records, T = tot.t, Q = tot.q, R = tot.r;
  const uint32_t H = d.h, FF = d.ffn;
  KC_CHECK(build_images(h));
  KC_TRY(cudaMemsetAsync(h->d_err, 0, sizeof(int), h->stream), "memset");
  KC_TRY(cudaMemsetAsync(ws.flags.p, 0, b.frames * 4ull, h->stream), "memset");
  float* x = P<float>(ws.x);
  float* qkv = P<float>(ws.qkv);
  if (T > 0) {
    ProfScope ps(h, kStEmbed);
    launch_embed(h, ws, b, x, T);
  }
  const float attn_scale = float(1.0 / std::sqrt(double(d.hd)));
  const int enc_m = 0, mix_m = 3 * int(d.enc), sel_m = mix_m + 5 * int(d.mix);
  if (attn_fusable(h) && d.enc > 0) KC_CHECK(attn_prepare(h, ws, T));
  for (uint32_t blk = 0; blk < d.enc && T > 0; blk++) {
    if (attn_fusable(h)) {  // q|k|v, attention and the residual in one kernel: q|k|v stay on chip
      ProfScope ps(h, kStEncAttnTc, 2.0 * T * H * 3 * H, 4.0 * T * (2 * H));
      KC_CHECK(tc_attn(h, ws, x, T, enc_m + 3 * blk, b.word_ids, b.word_alpha, attn_scale));
    } else {
      {
        ProfScope ps(h, kStEncGemm, 2.0 * T * H * 3 * H, 4.0 * T * (H + 3 * H));
        KC_CHECK(tc_gemm<kc::tc::kEpiStore>(h, x, T, enc_m + 3 * blk, qkv));
      }
      {
        ProfScope ps(h, kStEncAttn);
        kc::LocalAttnFastArgs la{qkv, x, P<uint32_t>(ws.rec_start), P<uint2>(ws.rec_meta), N, attn_scale,
                                 P<uint32_t>(ws.tok_recpos), b.word_alpha != 0.0f ? b.word_ids : nullptr,
                                 b.word_alpha};
        kc::k_local_attn_fast<<<unsigned((N + kc::kLaWarps - 1) / kc::kLaWarps), kc::kLaWarps * 32, 0,
                                h->stream>>>(la);
        h->launches++;
      }
    }
    if (ffn_fusable(h)) {  // W1, ReLU, W2 and the residual in one kernel: h1 stays on chip
      ProfScope ps(h, kStEncFfn, 4.0 * T * H * FF, 4.0 * T * (2 * H));
      KC_CHECK(tc_ffn(h, x, T, enc_m + 3 * blk + 1, enc_m + 3 * blk + 2));
    } else {
      {
        ProfScope ps(h, kStEncGemm, 2.0 * T * H * FF, 4.0 * T * (H + FF));
        KC_CHECK(tc_gemm<kc::tc::kEpiRelu>(h, x, T, enc_m + 3 * blk + 1, qkv));
      }
      {
        ProfScope ps(h, kStEncGemm, 2.0 * T * H * FF, 4.0 * T * (FF + 2 * H));
        KC_CHECK(tc_gemm<kc::tc::kEpiResid>(h, qkv, T, enc_m + 3 * blk + 2, x));
      }
    }
  }
  {
    ProfScope ps(h, kStPool);
    kc::PoolFastArgs pa{x, h->w + d.off_pool, P<uint32_t>(ws.rec_start), P<uint2>(ws.rec_meta),
                        P<uint32_t>(ws.rec_row), N, float(1.0 / std::sqrt(double(H))), P<float>(ws.bk),
                        P<float>(ws.bv), P<float>(ws.qstate)};
    kc::k_pool_fast<<<unsigned((N + 7) / 8), 256, 0, h->stream>>>(pa);
    h->launches++;
  }
  // the bank-side projections as planes products: bk once through the
  // selector's Wk (plane 0 of ws.sk, where the selector reads it) and every
  // block's Wk (planes 1..), bv once through every block's Wv (planes of ws.mv)
  const bool planes = !h->kplanes.empty() && Q > 0;
  if (planes) {
    ProfScope ps(h, kStMixer);
    KC_TRY(ensure(h, ws.sk, h->kplanes.size() * R * H * 4), "workspace");
    KC_TRY(ensure(h, ws.mv, h->vplanes.size() * R * H * 4), "workspace");
    KC_CHECK(tc_gemm_planes(h, P<float>(ws.bk), R, h->kplanes, P<float>(ws.sk)));
    KC_CHECK(tc_gemm_planes(h, P<float>(ws.bv), R, h->vplanes, P<float>(ws.mv)));
  }
  if (Q > 0) {
    ProfScope ps(h, kStMixer);
    for (uint32_t blk = 0; blk < d.mix; blk++) {
      const int m0 = mix_m + 5 * int(blk);
      KC_CHECK(tc_gemm<kc::tc::kEpiStore>(h, P<float>(ws.qstate), Q, m0, P<float>(ws.mq)));
      float* mk = planes ? P<float>(ws.sk) + (1 + blk) * R * H : P<float>(ws.mk);
      float* mv = planes ? P<float>(ws.mv) + blk * R * H : P<float>(ws.mv);
      if (!planes) {
        KC_CHECK(tc_gemm<kc::tc::kEpiStore>(h, P<float>(ws.bk), R, m0 + 1, mk));
        KC_CHECK(tc_gemm<kc::tc::kEpiStore>(h, P<float>(ws.bv), R, m0 + 2, mv));
      }
      if (tot.max_r <= uint32_t(kc::kCsMaxBank)) {  // every bank fits the one-pass kernel's score buffer
        const int chunks = int((std::max<uint32_t>(tot.max_q, 1) + kc::kCsChunk - 1) / kc::kCsChunk);
        kc::CrossAttnSmallArgs ca{P<float>(ws.mq),       mk,                      mv,
                                  P<float>(ws.qstate),   P<uint64_t>(ws.q_off),   P<uint64_t>(ws.r_off),
                                  kc::kCsChunk,          chunks,                  cross_small_half(tot.max_r),
                                  attn_scale};
        kc::k_cross_attn_small<<<b.frames * unsigned(chunks), kc::kCsThreads, cross_small_smem(tot.max_r),
                                 h->stream>>>(ca);
      } else {
        const CrossShape cs = cross_shape(tot.max_r);
        const int chunks = int((std::max<uint32_t>(tot.max_q, 1) + kc::kCaChunk - 1) / kc::kCaChunk);
        kc::CrossAttnFrameArgs ca{P<float>(ws.mq),       mk,                    mv,
                                  P<float>(ws.qstate),   P<uint64_t>(ws.q_off), P<uint64_t>(ws.r_off),
                                  chunks,                cs.kb,                 cs.half,
                                  attn_scale};
        kc::k_cross_attn_frame<<<b.frames * unsigned(chunks), kc::kCaThreads, cs.smem, h->stream>>>(ca);
      }
      h->launches++;
      KC_CHECK(tc_gemm<kc::tc::kEpiRelu>(h, P<float>(ws.qstate), Q, m0 + 3, P<float>(ws.mh)));
      KC_CHECK(tc_gemm<kc::tc::kEpiResid>(h, P<float>(ws.mh), Q, m0 + 4, P<float>(ws.qstate)));
    }
  }
  if (Q > 0) {
    ProfScope ps(h, kStSelector);
    KC_CHECK(tc_gemm<kc::tc::kEpiStore>(h, P<float>(ws.qstate), Q, sel_m, P<float>(ws.sq)));
    if (!planes) KC_CHECK(tc_gemm<kc::tc::kEpiStore>(h, P<float>(ws.bk), R, sel_m + 1, P<float>(ws.sk)));
    launch_select_fast(h, ws, b, tot);
  }
  KC_TRY(cudaGetLastError(), "launch");
  return KC_OK;
}

// Takes up the audit of the last recomputation: the largest ratio of a
// fast score's distance from its exact score to the margin B that the
// selector allowed it. Above 1 the margin was too small for this data: the
// violation is counted and later batches run with four times the margin.
void audit_collect(kc_handle* h) {
  if (!h->audit_pending) return;
  wait_stream(h);
  h->audit_pending = false;
  const float r = *h->h_audit;
  h->prof.cert_audit_max = std::max(h->prof.cert_audit_max, double(r));
  if (r > 1.0f) {
    h->prof.cert_audit_violations++;
    h->kappa_mul = std::min(h->kappa_mul * 4.0f, 65536.0f);
  }
}

// Recompute on the exact path every frame the fast selector could not
// certify (or all of them after a split overflow), then scatter the exact
// p blocks and indices into the batch's outputs.
kc_status certify(kc_handle* h, Workspace& ws, const DevBatch& b, const kc::FrameTotals& tot) {
  const uint32_t F = b.frames;
  audit_collect(h);
  // one readback: the flags and, per frame, its tokens, questions and bank
  // rows, from which the host sizes the sub-batch and knows its totals
  if (h->h_flags_cap < F) {
    if (h->h_flags_pinned) cudaFreeHost(h->h_flags_pinned);
    h->h_flags_pinned = nullptr;
    h->h_flags_cap = 0;
    KC_TRY(cudaMallocHost(&h->h_flags_pinned, F * 20ull), "pinned");  // flags, t, q, r, then the list
    h->h_flags_cap = F;
  }
  uint32_t* hf = h->h_flags_pinned;
  KC_TRY(cudaMemcpyAsync(hf, ws.flags.p, F * 4ull, cudaMemcpyDeviceToHost, h->stream), "readback");
  KC_TRY(cudaMemcpyAsync(hf + F, ws.frame_t.p, F * 4ull, cudaMemcpyDeviceToHost, h->stream), "readback");
  KC_TRY(cudaMemcpyAsync(hf + 2 * F, ws.frame_q.p, F * 4ull, cudaMemcpyDeviceToHost, h->stream), "readback");
  KC_TRY(cudaMemcpyAsync(hf + 3 * F, ws.frame_r.p, F * 4ull, cudaMemcpyDeviceToHost, h->stream), "readback");
  KC_TRY(cudaMemcpyAsync(h->h_err, h->d_err, sizeof(int), cudaMemcpyDeviceToHost, h->stream), "readback");
  KC_TRY(wait_stream(h), "certify");
  const int e = *h->h_err;
  if (e & kc::tc::kErrTimeout)
    return fail(h, KC_ERR_TIMEOUT, "a tensor-core pipeline wait expired; the batch was not completed");
  const bool all = e & kc::tc::kErrOverflow;
  h->last_overflow = all;
  if (all && h->sa > -24) h->sa -= 6;  // later batches split at a smaller scale
  uint32_t* list = hf + 4 * F;  // pinned, so its upload is asynchronous
  uint32_t n = 0;
  kc::FrameTotals sub_tot{};
  uint64_t nrec = 0;
  for (uint32_t f = 0; f < F; f++) {
    if (!all && !hf[f]) continue;
    list[n++] = f;
    const uint64_t t = hf[F + f], q = hf[2 * F + f], r = hf[3 * F + f];
    sub_tot.t += t; sub_tot.q += q; sub_tot.r += r; sub_tot.p += q * r;
    sub_tot.max_q = std::max(sub_tot.max_q, uint32_t(q));
    sub_tot.max_r = std::max(sub_tot.max_r, uint32_t(r));
    nrec += q + r;  // every record of a frame is a question or a bank row
  }
  if (n == 0 || tot.q == 0) return KC_OK;
  ProfScope ps(h, kStFallback);
  h->prof.fallback_frames += n;
  const uint64_t nq = sub_tot.q, np = sub_tot.p;
  Workspace& fb = h->ws_fb;
  KC_TRY(ensure(h, fb.list, n * 4ull), "workspace");
  KC_TRY(ensure(h, fb.rec_off, (n + 1) * 8ull), "workspace");
  KC_TRY(ensure(h, fb.uniforms, (n + 1) * 8ull), "workspace");  // sub question offsets
  KC_TRY(cudaMemcpyAsync(fb.list.p, list, n * 4ull, cudaMemcpyHostToDevice, h->stream), "upload");
  KC_TRY(ensure(h, fb.rows_val, (n + 1) * 8ull), "workspace");  // sub p offsets, for an explicit mask
  kc::k_fallback_offsets<<<1, 1024, 0, h->stream>>>(P<uint32_t>(fb.list), n, b.rec_off, P<uint64_t>(ws.q_off),
                                                    P<uint64_t>(ws.p_off), P<uint64_t>(fb.rec_off),
                                                    P<uint64_t>(fb.uniforms), P<uint64_t>(fb.rows_val));
  h->launches++;
  // the sub question offsets live in fb.uniforms until the gather; move them
  KC_TRY(ensure(h, fb.rows_off, (n + 1) * 8ull), "workspace");
  KC_TRY(cudaMemcpyAsync(fb.rows_off.p, fb.uniforms.p, (n + 1) * 8ull, cudaMemcpyDeviceToDevice, h->stream), "copy");
  KC_TRY(ensure(h, fb.token_ids, nrec * 32), "workspace");
  KC_TRY(ensure(h, fb.field_roles, nrec * 32), "workspace");
  KC_TRY(ensure(h, fb.schema_ids, nrec * 4), "workspace");
  KC_TRY(ensure(h, fb.band_ids, nrec * 4), "workspace");
  KC_TRY(ensure(h, fb.schema_allow, nq * 32 + 32), "workspace");
  KC_TRY(ensure(h, fb.band_allow, nq * 4 + 4), "workspace");
  KC_TRY(ensure(h, fb.uniforms, nq * 8 + 8), "workspace");
  const bool words = b.word_ids && b.word_alpha != 0.0f;
  if (words) KC_TRY(ensure(h, fb.word_ids, nrec * 32), "workspace");
  if (b.mask) {
    KC_TRY(ensure(h, fb.mask, np * 4 + 4), "workspace");
    kc::k_fallback_mask<<<n, 256, 0, h->stream>>>(P<uint32_t>(fb.list), P<uint64_t>(ws.p_off),
                                                  P<uint64_t>(fb.rows_val), b.mask, P<float>(fb.mask));
    h->launches++;
  }
  kc::k_fallback_gather<<<n, 256, 0, h->stream>>>(
      P<uint32_t>(fb.list), b.rec_off, P<uint64_t>(ws.q_off), P<uint64_t>(fb.rec_off), P<uint64_t>(fb.rows_off),
      b.token_ids, b.field_roles, b.schema_ids, b.band_ids, b.schema_allow, b.band_allow, b.uniforms,
      words ? b.word_ids : nullptr, P<uint32_t>(fb.token_ids), P<uint32_t>(fb.field_roles),
      P<uint32_t>(fb.schema_ids), P<uint32_t>(fb.band_ids), P<uint32_t>(fb.schema_allow),
      P<uint32_t>(fb.band_allow), P<double>(fb.uniforms), words ? P<uint32_t>(fb.word_ids) : nullptr);
  h->launches++;
  DevBatch sub;
  sub.frames = n; sub.records = nrec; sub.rec_off = P<uint64_t>(fb.rec_off);
  sub.token_ids = P<uint32_t>(fb.token_ids); sub.field_roles = P<uint32_t>(fb.field_roles);
  sub.schema_ids = P<uint32_t>(fb.schema_ids); sub.band_ids = P<uint32_t>(fb.band_ids);
  sub.schema_allow = b.schema_allow ? P<uint32_t>(fb.schema_allow) : nullptr;
  sub.band_allow = b.band_allow ? P<uint32_t>(fb.band_allow) : nullptr;
  sub.uniforms = b.uniforms ? P<double>(fb.uniforms) : nullptr;
  sub.word_ids = words ? P<uint32_t>(fb.word_ids) : nullptr;
  sub.word_alpha = b.word_alpha;
  if (b.mask) { sub.mask = P<float>(fb.mask); sub.mask_len = np; }
  KC_CHECK(pack_batch(h, fb, sub, &sub_tot, &sub_tot));  // the totals are known: no readback
  KC_CHECK(forward_exact(h, fb, sub, sub_tot, false));
  // audit the margin on the recomputed frames: the fast scores against the exact ones
  KC_TRY(cudaMemsetAsync(h->d_audit, 0, sizeof(float), h->stream), "memset");
  const dim3 agrid(n, (std::max<uint32_t>(sub_tot.max_r, 1) + kc::kAuKeys - 1) / kc::kAuKeys,
                   (std::max<uint32_t>(sub_tot.max_q, 1) + kc::kAuChunk - 1) / kc::kAuChunk);
  kc::k_cert_audit<<<agrid, 256, kc::kAuSmem, h->stream>>>(P<uint32_t>(fb.list), P<uint64_t>(ws.q_off), P<uint64_t>(ws.r_off),
                                             P<uint64_t>(fb.q_off), P<uint64_t>(fb.r_off), P<float>(ws.sq),
                                             P<float>(ws.sk), P<float>(fb.sq), P<float>(fb.sk), P<float>(ws.nq),
                                             P<float>(ws.nk), P<float>(ws.kappa),
                                             float(1.0 / std::sqrt(double(h->d.h))),
                                             1.0 / std::sqrt(double(h->d.h)),
                                             reinterpret_cast<unsigned*>(h->d_audit));
  h->launches++;
  KC_TRY(cudaMemcpyAsync(h->h_audit, h->d_audit, sizeof(float), cudaMemcpyDeviceToHost, h->stream), "readback");
  h->audit_pending = true;
  h->prof.cert_audit_frames += n;
  kc::k_fallback_scatter<<<dim3(n, 32), 256, 0, h->stream>>>(P<uint32_t>(fb.list), P<uint64_t>(ws.p_off),
                                                   P<uint64_t>(ws.q_off), P<uint64_t>(fb.p_off),
                                                   P<uint64_t>(fb.q_off), P<float>(fb.p), P<uint32_t>(fb.index),
                                                   P<float>(ws.p), P<uint32_t>(ws.index));
  h->launches++;
  KC_TRY(cudaGetLastError(), "launch");
  return KC_OK;
}

// Pack, then encode (+ select) at the handle's precision. *tot receives the
// batch totals.
kc_status run_batch(kc_handle* h, const DevBatch& b, bool encode_only, kc::FrameTotals* tot_out) {
  kc::FrameTotals tot;
  KC_CHECK(pack_batch(h, h->ws, b, &tot));
  if (b.mask && tot.p > b.mask_len)
    return fail(h, KC_ERR_INVALID_ARG, "the selection mask is smaller than the batch's sum of Q_f * R_f");
  if (encode_only || h->precision == KC_PRECISION_EXACT) {
    KC_CHECK(forward_exact(h, h->ws, b, tot, encode_only));
  } else {
    KC_CHECK(forward_fast(h, h->ws, b, tot));
    if (h->precision == KC_PRECISION_CERTIFIED) KC_CHECK(certify(h, h->ws, b, tot));
  }
  *tot_out = tot;
  return KC_OK;
}

kc_status check_config(const kc_config* c) {
  if (!c) return fail(nullptr, KC_ERR_INVALID_ARG, "config is null");
  if (c->hidden_size != KC_H || c->head_count != KC_HEADS || c->head_dim != KC_HEAD_DIM)
    return fail(nullptr, KC_ERR_CAPACITY, "hiddenSize/headCount/headDim must be 128/4/32 (the kernels' geometry)");
  if (c->ffn_size == 0 || c->ffn_size % 128 != 0 || c->ffn_size > 1024)
    return fail(nullptr, KC_ERR_CAPACITY, "ffnSize must be a multiple of 128 up to 1024");
  if (c->pos_space < KC_RW || c->stream_space < 2 || c->band_space == 0 || c->schema_space == 0 ||
      c->token_space == 0 || c->field_space == 0)
    return fail(nullptr, KC_ERR_INVALID_ARG, "embedding table sizes are too small for the frame ABI");
  if (!c->token_rows || c->token_rows_len == 0)
    return fail(nullptr, KC_ERR_INVALID_ARG, "tokenRows is empty: a session supplies its own vocabulary");
  return KC_OK;
}

bool weights_ok(const Dims& d, const kc_weights_view* w) {
  if (!w || !w->embeddings || !w->pool || !w->selector_wq || !w->selector_wk || !w->value_head_wv) return false;
  if (d.route && !w->decision_head_wh) return false;
  if ((d.enc && !w->enc) || (d.mix && !w->mixer)) return false;
  for (uint32_t b = 0; b < d.enc; b++)
    if (!w->enc[b].wq || !w->enc[b].wk || !w->enc[b].wv || !w->enc[b].w1 || !w->enc[b].w2) return false;
  for (uint32_t b = 0; b < d.mix; b++)
    if (!w->mixer[b].wq || !w->mixer[b].wk || !w->mixer[b].wv || !w->mixer[b].w1 || !w->mixer[b].w2) return false;
  return true;
}

kc_status upload_blocks(kc_handle* h, const kc_block_view* blocks, uint32_t n, uint64_t base) {
  const Dims& d = h->d;
  const uint64_t hh = uint64_t(d.h) * d.h, fh = uint64_t(d.ffn) * d.h;
  for (uint32_t b = 0; b < n; b++) {
    float* dst = h->w + base + d.block * b;
    KC_TRY(cudaMemcpyAsync(dst, blocks[b].wq, hh * 4, cudaMemcpyHostToDevice, h->stream), "sync");
    KC_TRY(cudaMemcpyAsync(dst + hh, blocks[b].wk, hh * 4, cudaMemcpyHostToDevice, h->stream), "sync");
    KC_TRY(cudaMemcpyAsync(dst + 2 * hh, blocks[b].wv, hh * 4, cudaMemcpyHostToDevice, h->stream), "sync");
    KC_TRY(cudaMemcpyAsync(dst + 3 * hh, blocks[b].w1, fh * 4, cudaMemcpyHostToDevice, h->stream), "sync");
    KC_TRY(cudaMemcpyAsync(dst + 3 * hh + fh, blocks[b].w2, fh * 4, cudaMemcpyHostToDevice, h->stream), "sync");
  }
  return KC_OK;
}

__global__ void k_scatter_rows(float* page, const float* vals, const uint32_t* offs, uint32_t n, uint32_t h) {
  const uint32_t r = blockIdx.x;
  if (r >= n) return;
  for (uint32_t i = threadIdx.x; i < h; i += blockDim.x) page[uint64_t(offs[r]) + i] = vals[uint64_t(r) * h + i];
}

kc_status do_sync(kc_handle* h, const kc_weights_view* w, const kc_changes* ch) {
  const Dims& d = h->d;
  if (!weights_ok(d, w)) return fail(h, KC_ERR_INVALID_ARG, "weights view is incomplete");
  auto put = [&](uint64_t off, const float* src, uint64_t n) -> kc_status {
    KC_TRY(cudaMemcpyAsync(h->w + off, src, n * 4, cudaMemcpyHostToDevice, h->stream), "sync");
    return KC_OK;
  };
  kc_status s = KC_OK;
  const uint64_t hh = uint64_t(d.h) * d.h;
  const bool all = ch == nullptr;
  if (all) {
    if ((s = put(0, w->embeddings, d.emb_elems))) return s;
  } else if (ch->embedding_rows_count) {
    const uint32_t n = ch->embedding_rows_count;
    std::vector<float> vals(uint64_t(n) * d.h);
    for (uint32_t i = 0; i < n; i++) {
      const uint32_t off = ch->embedding_rows[i];
      if (uint64_t(off) + d.h > d.emb_elems) return fail(h, KC_ERR_INVALID_ARG, "embedding row outside the page");
      memcpy(&vals[uint64_t(i) * d.h], w->embeddings + off, d.h * 4);
    }
    KC_TRY(ensure(h, h->ws.rows_val, vals.size() * 4), "workspace");
    KC_TRY(ensure(h, h->ws.rows_off, n * 4ull), "workspace");
    KC_TRY(cudaMemcpyAsync(h->ws.rows_val.p, vals.data(), vals.size() * 4, cudaMemcpyHostToDevice, h->stream), "sync");
    KC_TRY(cudaMemcpyAsync(h->ws.rows_off.p, ch->embedding_rows, n * 4ull, cudaMemcpyHostToDevice, h->stream), "sync");
    k_scatter_rows<<<n, 128, 0, h->stream>>>(h->w, P<float>(h->ws.rows_val), P<uint32_t>(h->ws.rows_off), n, d.h);
    h->launches++;
  }
  if (all || ch->blocks) {
    if ((s = upload_blocks(h, w->enc, d.enc, d.off_enc))) return s;
    if ((s = upload_blocks(h, w->mixer, d.mix, d.off_mixer))) return s;
  }
  if (all || ch->pool)
    if ((s = put(d.off_pool, w->pool, 2ull * d.h))) return s;
  if (all || ch->selector) {
    if ((s = put(d.off_swq, w->selector_wq, hh))) return s;
    if ((s = put(d.off_swk, w->selector_wk, hh))) return s;
  }
  if ((all || ch->decision_head) && d.route)
    if ((s = put(d.off_dec, w->decision_head_wh, uint64_t(d.route) * 3 * d.h))) return s;
  if (all || ch->value_head)
    if ((s = put(d.off_val, w->value_head_wv, 3ull * d.h))) return s;
  // max |W| of every tensor-core matrix whose values moved (sets its split scale)
  const bool blocks = all || ch->blocks, sel = all || ch->selector;
  if (blocks || sel) {
    auto amax = [](const float* a, uint64_t n, float m) {
      for (uint64_t i = 0; i < n; i++) m = std::max(m, std::fabs(a[i]));
      return m;
    };
    const uint64_t fh = uint64_t(d.ffn) * d.h;
    size_t i = 0;
    for (uint32_t b = 0; b < d.enc; b++, i += 3) {
      if (!blocks) continue;
      const kc_block_view& bv = w->enc[b];
      h->mat_max[i] = amax(bv.wk, hh, amax(bv.wv, hh, amax(bv.wq, hh, 0.f)));
      h->mat_max[i + 1] = amax(bv.w1, fh, 0.f);
      h->mat_max[i + 2] = amax(bv.w2, fh, 0.f);
    }
    for (uint32_t b = 0; b < d.mix; b++, i += 5) {
      if (!blocks) continue;
      const kc_block_view& bv = w->mixer[b];
      h->mat_max[i] = amax(bv.wq, hh, 0.f);
      h->mat_max[i + 1] = amax(bv.wk, hh, 0.f);
      h->mat_max[i + 2] = amax(bv.wv, hh, 0.f);
      h->mat_max[i + 3] = amax(bv.w1, fh, 0.f);
      h->mat_max[i + 4] = amax(bv.w2, fh, 0.f);
    }
    if (sel) {
      h->mat_max[i] = amax(w->selector_wq, hh, 0.f);
      h->mat_max[i + 1] = amax(w->selector_wk, hh, 0.f);
    }
    const size_t nf = h->mats.size() / 2;  // a transposed matrix has its original's largest entry
    const size_t nsel = nf - 2;            // the selector's two matrices end each half
    for (size_t j = 0; j < nf; j++) {
      h->mat_max[nf + j] = h->mat_max[j];
      if (j < nsel ? blocks : sel) h->mat_dirty[j] = h->mat_dirty[nf + j] = h->oz_dirty[j] = h->oz_dirty[nf + j] = 1;
    }
    h->wt_blocks_dirty |= blocks;
    h->wt_sel_dirty |= sel;
  }
  KC_TRY(cudaStreamSynchronize(h->stream), "sync");
  return KC_OK;
}

template <typename T>
kc_status stage(kc_handle* h, DevBuf& buf, const T* src, uint64_t n) {
  KC_TRY(ensure(h, buf, n * sizeof(T)), "workspace");
  if (n) KC_TRY(cudaMemcpyAsync(buf.p, src, n * sizeof(T), cudaMemcpyHostToDevice, h->stream), "upload");
  return KC_OK;
}

// compileActiveFrame's record walk (masks.ts:73-74): the active list in
// order, ending at the first unoccupied entry. Active records are compacted
// into a one-frame batch staged on the device; slot numbers only name
// positions, so the forward is unchanged. *q and *r count the frame's
// questions and bank records.
kc_status stage_frame(kc_handle* h, const kc_frame_view* frame, DevBatch& b, uint32_t* q_out, uint32_t* r_out) {
  if (!frame || !frame->token_ids || !frame->field_roles || !frame->schema_ids || !frame->band_ids)
    return fail(h, KC_ERR_INVALID_ARG, "frame view is incomplete");
  if (frame->slots == 0) return fail(h, KC_ERR_INVALID_ARG, "a frame with no records has nothing to think about");
  const uint32_t slots = frame->slots;
  std::vector<uint32_t> act;
  act.reserve(slots);
  for (uint32_t i = 0; i < slots; i++) {
    const uint32_t s = frame->active_record_indices ? frame->active_record_indices[i] : i;
    if (s == KC_INVALID || s >= slots) break;
    act.push_back(s);
  }
  const uint32_t n = uint32_t(act.size());
  if (n == 0) return fail(h, KC_ERR_INVALID_ARG, "a frame with no records has nothing to think about");
  std::vector<uint32_t> tok(n * 8ull), role(n * 8ull), sch(n), bnd(n);
  uint32_t q = 0;
  for (uint32_t i = 0; i < n; i++) {
    const uint32_t s = act[i];
    memcpy(&tok[i * 8ull], frame->token_ids + s * 8ull, 32);
    memcpy(&role[i * 8ull], frame->field_roles + s * 8ull, 32);
    sch[i] = frame->schema_ids[s];
    bnd[i] = frame->band_ids[s];
    q += bnd[i] == KC_QUERY_BAND;
  }
  const uint64_t off[2] = {0, n};
  kc_status s;
  Workspace& ws = h->ws;
  if ((s = stage(h, ws.rec_off, off, 2)) || (s = stage(h, ws.token_ids, tok.data(), tok.size())) ||
      (s = stage(h, ws.field_roles, role.data(), role.size())) || (s = stage(h, ws.schema_ids, sch.data(), n)) ||
      (s = stage(h, ws.band_ids, bnd.data(), n)))
    return s;
  b.frames = 1; b.records = n; b.rec_off = P<uint64_t>(ws.rec_off);
  b.token_ids = P<uint32_t>(ws.token_ids); b.field_roles = P<uint32_t>(ws.field_roles);
  b.schema_ids = P<uint32_t>(ws.schema_ids); b.band_ids = P<uint32_t>(ws.band_ids);
  *q_out = q;
  *r_out = n - q;
  return KC_OK;
}

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

// The backward of every frame of a packed batch (backward.cuh), after an
// exact forward that saves what the backward reads. `sel`, `targets`,
// `valence` are device arrays or null. Results stay in h->bw and ws.p.
kc_status backward_batch(kc_handle* h, const DevBatch& b, const float* sel, const uint32_t* targets,
                         const double* valence, kc::FrameTotals* tot_out, bool exact) {
  // The GEMMs run on the tensor cores unless the handle or the caller asks
  // for the oracle's arithmetic; a split overflow reruns the batch exactly.
  const bool tc = !exact && h->precision != KC_PRECISION_EXACT;
  const Dims& d = h->d;
  Workspace& ws = h->ws;
  BackWs& bw = h->bw;
  kc::FrameTotals tot;
  KC_CHECK(pack_batch(h, ws, b, &tot));
  const uint32_t F = b.frames;
  const uint64_t N = b.records, T = tot.t, Q = tot.q, R = tot.r, PP = tot.p;
  const uint64_t H = d.h, FF = d.ffn;
  auto need = [&](DevBuf& buf, uint64_t bytes) { return ensure(h, buf, bytes); };
  KC_TRY(need(bw.mask, PP * 4), "workspace");
  KC_TRY(need(bw.enc_qkv, uint64_t(d.enc) * T * 3 * H * 4), "workspace");
  KC_TRY(need(bw.enc_p, uint64_t(d.enc) * T * 32 * 4), "workspace");
  KC_TRY(need(bw.enc_h1, uint64_t(d.enc) * T * FF * 4), "workspace");
  KC_TRY(need(bw.mix_q, uint64_t(d.mix) * Q * H * 4), "workspace");
  KC_TRY(need(bw.mix_k, uint64_t(d.mix) * R * H * 4), "workspace");
  KC_TRY(need(bw.mix_v, uint64_t(d.mix) * R * H * 4), "workspace");
  KC_TRY(need(bw.mix_p, uint64_t(d.mix) * 4 * PP * 4), "workspace");
  KC_TRY(need(bw.mix_h1, uint64_t(d.mix) * Q * FF * 4), "workspace");
  KC_TRY(need(bw.gather, Q * H * 4), "workspace");
  KC_TRY(need(bw.offered, Q * H * 4), "workspace");
  KC_TRY(need(bw.n_allowed, Q * 4), "workspace");
  KC_TRY(need(bw.pred, Q * 4), "workspace");
  KC_TRY(need(bw.dpred, Q * 4), "workspace");
  KC_TRY(need(bw.loss, F * 8ull), "workspace");
  KC_TRY(need(bw.dwv, F * 3 * H * 4), "workspace");
  KC_TRY(need(bw.dquery, Q * H * 4), "workspace");
  KC_TRY(need(bw.dig, Q * H * 4), "workspace");
  KC_TRY(need(bw.dag, Q * H * 4), "workspace");
  KC_TRY(need(bw.dscore, PP * 4), "workspace");
  KC_TRY(need(bw.dqp, Q * H * 4), "workspace");
  KC_TRY(need(bw.dkp, R * H * 4), "workspace");
  KC_TRY(need(bw.dbk, R * H * 4), "workspace");
  KC_TRY(need(bw.dbv, R * H * 4), "workspace");
  KC_TRY(need(bw.dswq, F * H * H * 4), "workspace");
  KC_TRY(need(bw.dswk, F * H * H * 4), "workspace");
  KC_TRY(need(bw.dh1, (Q > T ? Q : T) * FF * 4), "workspace");
  KC_TRY(need(bw.ads, 4 * PP * 4), "workspace");
  KC_TRY(need(bw.mdq, Q * H * 4), "workspace");
  KC_TRY(need(bw.mdk, R * H * 4), "workspace");
  KC_TRY(need(bw.mdv, R * H * 4), "workspace");
  KC_TRY(need(bw.tok_ds, T * 16), "workspace");
  KC_TRY(need(bw.dfs, T * H * 4), "workspace");
  KC_TRY(need(bw.dpool, F * 2 * H * 4), "workspace");
  KC_TRY(need(bw.edqkv, T * 3 * H * 4), "workspace");
  KC_TRY(ensure(h, ws.gather, Q * H * 4), "workspace");
  KC_CHECK(build_transposes(h));
  const float* wt = P<float>(h->wt);
  kc::BatchGeo geo{P<uint32_t>(ws.query_frame), P<uint32_t>(ws.bank_frame), P<uint64_t>(ws.q_off),
                   P<uint64_t>(ws.r_off), P<uint64_t>(ws.p_off)};
  // the selection: given, from the batch's rule, or open
  const float* mask = P<float>(bw.mask);
  if (sel) {
    mask = sel;
  } else if (b.schema_allow && Q) {
    kc::RuleMaskArgs ra{geo, b.schema_allow, b.band_allow, P<uint32_t>(ws.bank_rec), b.schema_ids, b.band_ids,
                        P<float>(bw.mask)};
    kc::k_rule_mask<<<unsigned(Q), 256, 0, h->stream>>>(ra);
    h->launches++;
  } else if (PP) {
    KC_TRY(cudaMemsetAsync(bw.mask.p, 0, PP * 4, h->stream), "memset");
  }
  if (Q) KC_TRY(cudaMemsetAsync(bw.gather.p, 0, Q * H * 4, h->stream), "memset");
  if (T) KC_TRY(cudaMemsetAsync(bw.dfs.p, 0, T * H * 4, h->stream), "memset");
  bw.frames = 0;
  bw.mask_used = mask;
  Saves sv{P<float>(bw.enc_qkv), P<float>(bw.enc_p), P<float>(bw.enc_h1), P<float>(bw.mix_q), P<float>(bw.mix_k),
           P<float>(bw.mix_v), P<float>(bw.mix_p), P<float>(bw.mix_h1), mask, P<float>(bw.gather)};
  if (tc) {
    KC_CHECK(build_images(h));
    KC_TRY(cudaMemsetAsync(h->d_err, 0, sizeof(int), h->stream), "memset");
  }
  KC_CHECK(forward_exact(h, ws, b, tot, false, &sv, tc));
  const int nf = int(h->mats.size() / 2);  // transposed matrices follow the forward ones
  const int sel_m = 3 * int(d.enc) + 5 * int(d.mix);

  const double h_scale = 1.0 / std::sqrt(double(H));
  const double attn_scale = 1.0 / std::sqrt(double(d.hd));
  const float* qout = P<float>(ws.qstate);
  const float* bk = P<float>(ws.bk);
  const float* bv = P<float>(ws.bv);
  const float* p = P<float>(ws.p);
  float* dquery = P<float>(bw.dquery);
  float* dbk = P<float>(bw.dbk);
  float* dbv = P<float>(bw.dbv);
  {
    ProfScope ps(h, kStSelector);
    if (Q) {
      kc::OfferedArgs oa{geo, mask, bv, qout, P<float>(bw.gather), h->w + d.off_val, P<float>(bw.offered),
                         P<uint32_t>(bw.n_allowed), P<float>(bw.pred)};
      kc::k_offered_pred<<<unsigned(Q), 128, 0, h->stream>>>(oa);
      h->launches++;
    }
    kc::k_value_loss<<<(F + 127) / 128, 128, 0, h->stream>>>(P<float>(bw.pred), valence, P<uint64_t>(ws.q_off), F,
                                                              P<float>(bw.dpred), P<double>(bw.loss));
    kc::k_value_wv<<<F, 384, 0, h->stream>>>(qout, P<float>(bw.gather), P<float>(bw.offered), P<float>(bw.dpred),
                                             P<uint64_t>(ws.q_off), P<float>(bw.dwv));
    h->launches += 2;
    if (Q) {
      kc::SelBackArgs sb{geo, p, bv, h->w + d.off_val, P<float>(bw.dpred), targets, dquery, P<float>(bw.dig),
                         P<float>(bw.dag), P<float>(bw.dscore)};
      kc::k_sel_back_scores<<<unsigned(Q), 256, size_t(tot.max_r) * 12, h->stream>>>(sb);
      kc::k_sel_back_dq<<<unsigned(Q), 128, 0, h->stream>>>(geo, P<float>(bw.dscore), P<float>(ws.sk), h_scale,
                                                           P<float>(bw.dqp));
      h->launches += 2;
    }
    if (R) {
      kc::SelBackKArgs sk{geo, P<float>(bw.dscore), p, mask, P<float>(ws.sq), P<float>(bw.dig), P<float>(bw.dag),
                          P<uint32_t>(bw.n_allowed), h_scale, P<float>(bw.dkp), dbv, uint32_t(R)};
      kc::k_sel_back_dk<<<unsigned((R + kc::kSelBackRows - 1) / kc::kSelBackRows), 128, 0, h->stream>>>(sk);
      h->launches++;
    }
    // dQuery = dQueryOut + dQProj·Wq; dBankKeys = dKProj·Wk (backward.ts:900-912)
    KC_CHECK(gemm<kc::kEpiResid>(h, tc, P<float>(bw.dqp), H, Q, nf + sel_m, wt + d.off_swq, H, dquery, H, H));
    KC_CHECK(gemm<kc::kEpiStore>(h, tc, P<float>(bw.dkp), H, R, nf + sel_m + 1, wt + d.off_swk, H, dbk, H, H));
    kc::k_weight_grad<<<dim3(F, H / 8), 256, 0, h->stream>>>(P<float>(bw.dqp), qout, P<uint64_t>(ws.q_off),
                                                             P<float>(bw.dswq));
    kc::k_weight_grad<<<dim3(F, H / 8), 256, 0, h->stream>>>(P<float>(bw.dkp), bk, P<uint64_t>(ws.r_off),
                                                             P<float>(bw.dswk));
    h->launches += 2;
  }
  // mixer blocks in reverse (backward.ts:925-941)
  if (Q) {
    ProfScope ps(h, kStMixer);
    for (int blk = int(d.mix) - 1; blk >= 0; blk--) {
      const uint64_t o = d.off_mixer + d.block * blk;
      const float* wT = wt + o;  // Wqᵀ, Wkᵀ, Wvᵀ [H,H], W1ᵀ [H,F], W2ᵀ [F,H]
      float* dh1 = P<float>(bw.dh1);
      const int m0 = nf + 3 * int(d.enc) + 5 * blk;
      KC_CHECK(gemm<kc::kEpiGate>(h, tc, dquery, H, Q, m0 + 4, wT + 3 * H * H + FF * H, H, dh1, FF, H,
                                  P<float>(bw.mix_h1) + blk * Q * FF));
      KC_CHECK(gemm<kc::kEpiResid>(h, tc, dh1, FF, Q, m0 + 3, wT + 3 * H * H, FF, dquery, H, FF));
      kc::CrossBackArgs cb{geo, dquery, P<float>(bw.mix_q) + blk * Q * H, P<float>(bw.mix_k) + blk * R * H,
                           P<float>(bw.mix_v) + blk * R * H, P<float>(bw.mix_p) + blk * 4 * PP, PP, tot.max_r,
                           attn_scale, P<float>(bw.ads), P<float>(bw.mdq), P<float>(bw.mdk), P<float>(bw.mdv)};
      kc::k_cross_attn_back_q<<<unsigned(Q), 128, size_t(tot.max_r) * 48, h->stream>>>(cb);
      h->launches++;
      if (R) {
        cb.rows = uint32_t(R);
        kc::k_cross_attn_back_kv<<<unsigned((R + kc::kCrossBackRows - 1) / kc::kCrossBackRows), 128, 0,
                                   h->stream>>>(cb);
        h->launches++;
      }
      KC_CHECK(gemm<kc::kEpiResid>(h, tc, P<float>(bw.mdq), H, Q, m0, wT, H, dquery, H, H));
      KC_CHECK(gemm<kc::kEpiResid>(h, tc, P<float>(bw.mdk), H, R, m0 + 1, wT + H * H, H, dbk, H, H));
      KC_CHECK(gemm<kc::kEpiResid>(h, tc, P<float>(bw.mdv), H, R, m0 + 2, wT + 2 * H * H, H, dbv, H, H));
    }
  }
  // pool backward (backward.ts:944-953)
  {
    ProfScope ps(h, kStPool);
    kc::PoolBackArgs pb{P<float>(ws.x), h->w + d.off_pool, P<uint32_t>(ws.rec_start), P<uint2>(ws.rec_meta),
                        P<uint32_t>(ws.rec_row), N, h_scale, dbk, dbv, dquery, P<float>(bw.dfs),
                        P<double>(bw.tok_ds)};
    kc::k_pool_back<<<unsigned((N + 7) / 8), 256, 0, h->stream>>>(pb);
    kc::PoolGradArgs pg{P<float>(ws.x), P<double>(bw.tok_ds), P<uint32_t>(ws.rec_start), P<uint2>(ws.rec_meta),
                        P<uint32_t>(ws.bank_rec), P<uint32_t>(ws.query_rec), P<uint64_t>(ws.r_off),
                        P<uint64_t>(ws.q_off), h_scale, P<float>(bw.dpool)};
    kc::k_pool_grad<<<F, 256, 0, h->stream>>>(pg);
    h->launches += 2;
  }
  // encoder blocks in reverse (backward.ts:956-968)
  float* dfs = P<float>(bw.dfs);
  for (int blk = int(d.enc) - 1; blk >= 0 && T > 0; blk--) {
    const uint64_t o = d.off_enc + d.block * blk;
    const float* wT = wt + o;
    float* dh1 = P<float>(bw.dh1);
    const int em = nf + 3 * blk;
    {
      ProfScope ps(h, kStEncGemm, 2.0 * T * H * FF, 4.0 * T * (H + 2 * FF));
      KC_CHECK(gemm<kc::kEpiGate>(h, tc, dfs, H, T, em + 2, wT + 3 * H * H + FF * H, H, dh1, FF, H,
                                  P<float>(bw.enc_h1) + blk * T * FF));
    }
    {
      ProfScope ps(h, kStEncGemm, 2.0 * T * H * FF, 4.0 * T * (FF + 2 * H));
      KC_CHECK(gemm<kc::kEpiResid>(h, tc, dh1, FF, T, em + 1, wT + 3 * H * H, FF, dfs, H, FF));
    }
    {
      ProfScope ps(h, kStEncAttn);
      kc::LocalBackArgs lb{P<float>(bw.enc_qkv) + blk * T * 3 * H, P<float>(bw.enc_p) + blk * T * 32, dfs,
                           P<uint32_t>(ws.rec_start), P<uint2>(ws.rec_meta), N, attn_scale, P<float>(bw.edqkv)};
      const unsigned grid = unsigned((N + kc::kLocalBackWarps - 1) / kc::kLocalBackWarps);
      if (tc)  // the tensor-core backward: the same chains in f32
        kc::k_local_attn_back<float><<<grid, kc::kLocalBackWarps * 32, kc::kLocalBackSmem, h->stream>>>(lb);
      else
        kc::k_local_attn_back<double><<<grid, kc::kLocalBackWarps * 32, kc::kLocalBackSmem, h->stream>>>(lb);
      h->launches++;
    }
    // dStates += dQ·Wq + dK·Wk + dV·Wv: three f32-rounded adds in the oracle's
    // order, or one product over [dQ | dK | dV] · [Wqᵀ | Wkᵀ | Wvᵀ]ᵀ on the tensor cores
    const float* e = P<float>(bw.edqkv);
    if (tc) {
      ProfScope ps(h, kStEncGemm, 2.0 * T * H * 3 * H, 4.0 * T * 5 * H);
      KC_CHECK(gemm<kc::kEpiResid>(h, tc, e, 3 * H, T, em, wT, 3 * H, dfs, H, 3 * H));
    } else {
      for (int part = 0; part < 3; part++) {
        ProfScope ps(h, kStEncGemm, 2.0 * T * H * H, 4.0 * T * 3 * H);
        KC_CHECK(dgemm_ld<kc::kEpiResid>(h, e + part * H, 3 * H, wT + part * H, dfs, T, H, H, nullptr, 3 * H));
      }
    }
  }
  KC_TRY(cudaGetLastError(), "backward launch");
  if (tc) {
    KC_TRY(cudaMemcpyAsync(h->h_err, h->d_err, sizeof(int), cudaMemcpyDeviceToHost, h->stream), "readback");
    KC_TRY(cudaStreamSynchronize(h->stream), "backward");
    const int e = *h->h_err;
    if (e & kc::tc::kErrTimeout) return fail(h, KC_ERR_TIMEOUT, "a tensor-core pipeline wait expired");
    if (e & kc::tc::kErrOverflow) return backward_batch(h, b, sel, targets, valence, tot_out, true);
  }
  bw.frames = F;
  *tot_out = tot;
  return KC_OK;
}

}  // namespace

extern "C" {

uint32_t kc_abi_version(void) { return KC_ABI_VERSION; }

kc_status kc_create(const kc_config* config, const kc_weights_view* weights, int device, kc_handle** out) {
  if (!out) return fail(nullptr, KC_ERR_INVALID_ARG, "out is null");
  *out = nullptr;
  kc_status s = check_config(config);
  if (s) return s;
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
    cudaGetLastError();
    return fail(nullptr, KC_ERR_NO_DEVICE, "no CUDA device");
  }
  if (device < 0 || device >= ndev) return fail(nullptr, KC_ERR_INVALID_ARG, "device index out of range");
  DeviceGuard dg(device);
  auto* h = new kc_handle();
  h->device = device;
  h->d = dims_of(config);
  {
    const char* nf = std::getenv("KC_NO_FUSION");
    h->fuse = !(nf && nf[0] && nf[0] != '0');
    const char* no = std::getenv("KC_NO_OZAKI");
    h->oz = !(no && no[0] && no[0] != '0');
    const char* cap = std::getenv("KC_OZAKI_LIST_CAP");
    if (cap && cap[0]) h->oz_cap = std::max(0ll, std::atoll(cap));
  }
  if (!weights_ok(h->d, weights)) {
    delete h;
    return fail(nullptr, KC_ERR_INVALID_ARG, "weights view is incomplete");
  }
  auto bail = [&](cudaError_t e, const char* what) {
    std::string m = std::string(what) + ": " + cudaGetErrorString(e);
    kc_destroy(h);
    return fail(nullptr, e == cudaErrorMemoryAllocation ? KC_ERR_CAPACITY : KC_ERR_CUDA, m);
  };
  cudaError_t e;
  if ((e = cudaStreamCreateWithFlags(&h->own, cudaStreamNonBlocking))) return bail(e, "stream");
  h->stream = h->own;
  if ((e = cudaMalloc(&h->w, h->d.total * 4))) return bail(e, "weights");
  h->token_rows_len = config->token_rows_len;
  h->token_rows_host.assign(config->token_rows, config->token_rows + config->token_rows_len);
  h->id_ok.resize(h->token_rows_len);
  for (uint32_t i = 0; i < h->token_rows_len; i++)
    h->id_ok[i] = uint8_t((h->token_rows_host[i] < h->d.token_space ? 1u : 0u) |
                          (h->token_rows_host[i] < h->d.field_space ? 2u : 0u));
  if ((e = cudaMalloc(&h->token_rows, uint64_t(h->token_rows_len) * 4))) return bail(e, "tokenRows");
  if ((e = cudaMemcpy(h->token_rows, config->token_rows, uint64_t(h->token_rows_len) * 4, cudaMemcpyHostToDevice)))
    return bail(e, "tokenRows");
  if ((e = cudaMallocHost(&h->h_tot, sizeof(kc::FrameTotals)))) return bail(e, "pinned");
  if ((e = cudaMallocHost(&h->h_err, sizeof(int)))) return bail(e, "pinned");
  if ((e = cudaMalloc(&h->d_err, sizeof(int)))) return bail(e, "error word");
  if ((e = cudaMallocHost(&h->h_oz_err, sizeof(int)))) return bail(e, "pinned");
  if ((e = cudaMalloc(&h->d_oz_word, 4 * sizeof(unsigned)))) return bail(e, "error word");
  if ((e = cudaMemset(h->d_oz_word, 0, 4 * sizeof(unsigned)))) return bail(e, "error word");
  if ((e = cudaMallocHost(&h->h_audit, sizeof(float)))) return bail(e, "pinned");
  if ((e = cudaMalloc(&h->d_audit, sizeof(float)))) return bail(e, "audit word");
  if ((e = cudaDeviceGetAttribute(&h->sms, cudaDevAttrMultiProcessorCount, device))) return bail(e, "attributes");
  h->mats = mat_list(h->d);
  {
    // KC_NO_PLANES=1 at kc_create: one product per bank-side projection (the
    // same bits; kept to check the planes products against)
    const char* np = std::getenv("KC_NO_PLANES");
    if (!(np && np[0] && np[0] != '0')) plan_planes(h);
  }
  h->mat_max.assign(h->mats.size(), 0.f);
  h->mat_dirty.assign(h->mats.size(), 1);
  h->oz_dirty.assign(h->mats.size(), 1);
  for (const Mat& m : h->mats)
    if (m.n % 128 || m.k % 64) {
      kc_destroy(h);
      return fail(nullptr, KC_ERR_CAPACITY, "tensor-core path needs matrix sizes in multiples of 128 x 64");
    }
  if ((e = cudaFuncSetAttribute(kc::tc::k_tc_gemm<kc::tc::kEpiStore>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                kc::tc::kSmemBytesT)) ||
      (e = cudaFuncSetAttribute(kc::tc::k_tc_gemm<kc::tc::kEpiRelu>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                kc::tc::kSmemBytesT)) ||
      (e = cudaFuncSetAttribute(kc::tc::k_tc_gemm<kc::tc::kEpiResid>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                kc::tc::kSmemBytesT)) ||
      (e = cudaFuncSetAttribute(kc::tc::k_tc_gemm<kc::tc::kEpiGate>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                kc::tc::kSmemBytesT)) ||
      (e = cudaFuncSetAttribute(kc::tc::k_tc_ffn, cudaFuncAttributeMaxDynamicSharedMemorySize, kc::tc::kFfnSmem)) ||
      (e = cudaFuncSetAttribute(kc::tc::k_tc_attn<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                kc::tc::kAtSmem)) ||
      (e = cudaFuncSetAttribute(kc::tc::k_tc_attn<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                kc::tc::kAtSmem)) ||
      (e = cudaFuncSetAttribute(kc::k_embed_exact, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(kc::kEmbedSmemMax))) ||
      (e = cudaFuncSetAttribute(kc::k_learn_plan, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(kc::kPlanSmem))) ||
      (e = cudaFuncSetAttribute(kc::k_cross_attn_frame, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(cross_shape(kc::kCaBlock).smem))) ||
      (e = cudaFuncSetAttribute(kc::k_cross_attn_small, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(cross_small_smem(kc::kCsMaxBank)))) ||
      (e = cudaFuncSetAttribute(kc::k_select_fast, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (96 << 10) + kc::kSelChunk * KC_H * 4)))
    return bail(e, "smem");
  if ((e = cudaFuncSetAttribute(kc::k_cross_attn_exact<16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(kc::xa_smem(16)))) ||
      (e = cudaFuncSetAttribute(kc::k_cross_attn_exact<8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(kc::xa_smem(8)))) ||
      (e = cudaFuncSetAttribute(kc::k_cross_attn_exact<4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(kc::xa_smem(4)))))
    return bail(e, "smem");
  if ((e = cudaFuncSetAttribute(kc::k_select_scores_fast, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(kc::kSsSmem)))) return bail(e, "smem");
  if ((e = cudaFuncSetAttribute(kc::k_cert_audit, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(kc::kAuSmem)))) return bail(e, "smem");
  if ((e = cudaFuncSetAttribute(kc::k_select_scores_exact, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(kc::kXsSmem)))) return bail(e, "smem");
  if ((e = cudaFuncSetAttribute(kc::k_select_exact, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(KC_MAX_BANK) * (8 + 4)))) return bail(e, "smem");
  if ((e = cudaFuncSetAttribute(kc::k_sel_back_scores, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(KC_MAX_BANK) * 12))) return bail(e, "smem");
  if ((e = cudaFuncSetAttribute(kc::k_cross_attn_back_q, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(KC_MAX_BANK) * 48)) ||
      (e = cudaFuncSetAttribute(kc::k_local_attn_back<double>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(kc::kLocalBackSmem))) ||
      (e = cudaFuncSetAttribute(kc::k_local_attn_back<float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(kc::kLocalBackSmem))))
    return bail(e, "smem");
  if ((e = cudaFuncSetAttribute(kc::oz::k_oz_gemm<kc::kEpiStore>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                kc::oz::kSmem)) ||
      (e = cudaFuncSetAttribute(kc::oz::k_oz_gemm<kc::kEpiRelu>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                kc::oz::kSmem)) ||
      (e = cudaFuncSetAttribute(kc::oz::k_oz_gemm<kc::kEpiResid>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                kc::oz::kSmem)) ||
      (e = cudaFuncSetAttribute(kc::oz::k_oz_gemm<kc::kEpiGate>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                kc::oz::kSmem)))
    return bail(e, "smem");
  s = do_sync(h, weights, nullptr);
  if (s) {
    std::string m = h->err;
    kc_destroy(h);
    return fail(nullptr, s, m);
  }
  *out = h;
  return KC_OK;
}

kc_status kc_sync(kc_handle* h, const kc_weights_view* weights, const kc_changes* changes) {
  if (!h) return fail(nullptr, KC_ERR_INVALID_ARG, "handle is null");
  std::lock_guard<std::mutex> lk(h->mu);
  h->ws_epoch++;  // the resident batch (kc_select_batch) is gone
  DeviceGuard dg(h->device);
  return do_sync(h, weights, changes);
}

kc_status kc_encode(kc_handle* h, const kc_frame_view* frame, float* query_output, float* bank_keys,
                    float* bank_values, uint32_t q_cap, uint32_t r_cap, uint32_t* q_out, uint32_t* r_out) {
  if (!h) return fail(nullptr, KC_ERR_INVALID_ARG, "handle is null");
  std::lock_guard<std::mutex> lk(h->mu);
  h->ws_epoch++;  // the resident batch (kc_select_batch) is gone
  DeviceGuard dg(h->device);
  uint32_t q = 0, r = 0;
  DevBatch b;
  kc_status s = stage_frame(h, frame, b, &q, &r);
  if (s) return s;
  if (q == 0) return fail(h, KC_ERR_INVALID_ARG, "the frame must contain at least one query record for the mixer");
  if (q > q_cap || r > r_cap) return fail(h, KC_ERR_CAPACITY, "output buffers are smaller than the frame's Q/R");
  Workspace& ws = h->ws;
  kc::FrameTotals tot;
  if ((s = run_batch(h, b, true, &tot))) return s;
  const uint64_t H = h->d.h;
  KC_TRY(cudaMemcpyAsync(query_output, ws.qstate.p, q * H * 4, cudaMemcpyDeviceToHost, h->stream), "readback");
  if (r) {
    KC_TRY(cudaMemcpyAsync(bank_keys, ws.bk.p, r * H * 4, cudaMemcpyDeviceToHost, h->stream), "readback");
    KC_TRY(cudaMemcpyAsync(bank_values, ws.bv.p, r * H * 4, cudaMemcpyDeviceToHost, h->stream), "readback");
  }
  KC_TRY(cudaStreamSynchronize(h->stream), "encode");
  prof_collect(h);
  if (q_out) *q_out = q;
  if (r_out) *r_out = r;
  return KC_OK;
}

kc_status kc_select(kc_handle* h, const kc_encoded_view* enc, const float* mask, const kc_mask_rule* rule,
                    const double* uniforms, float* p, uint32_t* index, float* gather) {
  if (!h) return fail(nullptr, KC_ERR_INVALID_ARG, "handle is null");
  std::lock_guard<std::mutex> lk(h->mu);
  h->ws_epoch++;  // the resident batch (kc_select_batch) is gone
  DeviceGuard dg(h->device);
  if (!enc || !enc->query_output || (enc->r && (!enc->bank_keys || !enc->bank_values)) || !p || !index)
    return fail(h, KC_ERR_INVALID_ARG, "select arguments are incomplete");
  if (rule && (!rule->schema_allow || !rule->band_allow || !rule->bank_schema_ids || !rule->bank_band_ids))
    return fail(h, KC_ERR_INVALID_ARG, "mask rule is incomplete");
  const uint32_t Q = enc->q, R = enc->r;
  if (Q == 0) return KC_OK;
  if (R > KC_MAX_BANK) return fail(h, KC_ERR_CAPACITY, "bank records exceed capacity");
  const uint64_t H = h->d.h;
  Workspace& ws = h->ws;
  // a one-frame view: every question belongs to frame 0
  const uint64_t r_off[2] = {0, R}, q_off[2] = {0, Q}, p_off[2] = {0, uint64_t(Q) * R};
  std::vector<uint32_t> qframe(Q, 0u), bank_rec(R);
  for (uint32_t j = 0; j < R; j++) bank_rec[j] = j;
  kc_status s;
  if ((s = stage(h, ws.r_off, r_off, 2)) || (s = stage(h, ws.q_off, q_off, 2)) || (s = stage(h, ws.p_off, p_off, 2)) ||
      (s = stage(h, ws.query_frame, qframe.data(), Q)) || (s = stage(h, ws.bank_rec, bank_rec.data(), R)) ||
      (s = stage(h, ws.qstate, enc->query_output, Q * H)) || (s = stage(h, ws.bk, enc->bank_keys, R * H)) ||
      (s = stage(h, ws.bv, enc->bank_values, R * H)))
    return s;
  if (mask && (s = stage(h, ws.mask, mask, uint64_t(Q) * R))) return s;
  if (rule) {
    if ((s = stage(h, ws.schema_allow, rule->schema_allow, Q * 8ull)) ||
        (s = stage(h, ws.band_allow, rule->band_allow, Q)) ||
        (s = stage(h, ws.bank_schema, rule->bank_schema_ids, R)) || (s = stage(h, ws.bank_band, rule->bank_band_ids, R)))
      return s;
  }
  if (uniforms && (s = stage(h, ws.uniforms, uniforms, Q))) return s;
  KC_TRY(ensure(h, ws.sq, Q * H * 4), "workspace");
  KC_TRY(ensure(h, ws.sk, R * H * 4), "workspace");
  KC_TRY(ensure(h, ws.p, uint64_t(Q) * R * 4), "workspace");
  KC_TRY(ensure(h, ws.index, Q * 4ull), "workspace");
  KC_TRY(ensure(h, ws.gather, Q * H * 4), "workspace");
  {
    ProfScope ps(h, kStSelector);
    dgemm<kc::kEpiStore>(h, P<float>(ws.qstate), h->w + h->d.off_swq, P<float>(ws.sq), Q, uint32_t(H), uint32_t(H));
    dgemm<kc::kEpiStore>(h, P<float>(ws.bk), h->w + h->d.off_swk, P<float>(ws.sk), R, uint32_t(H), uint32_t(H));
    kc::SelectArgs sa{};
    sa.sq = P<float>(ws.sq); sa.sk = P<float>(ws.sk); sa.bank_values = P<float>(ws.bv);
    sa.query_frame = P<uint32_t>(ws.query_frame); sa.r_off = P<uint64_t>(ws.r_off);
    sa.q_off = P<uint64_t>(ws.q_off); sa.p_off = P<uint64_t>(ws.p_off);
    sa.mask = mask ? P<float>(ws.mask) : nullptr;
    sa.schema_allow = rule ? P<uint32_t>(ws.schema_allow) : nullptr;
    sa.band_allow = rule ? P<uint32_t>(ws.band_allow) : nullptr;
    sa.bank_rec = P<uint32_t>(ws.bank_rec);
    sa.schema_ids = rule ? P<uint32_t>(ws.bank_schema) : nullptr;
    sa.band_ids = rule ? P<uint32_t>(ws.bank_band) : nullptr;
    sa.uniforms = uniforms ? P<double>(ws.uniforms) : nullptr;
    sa.max_r = R; sa.scale = 1.0 / std::sqrt(double(H));
    sa.p = P<float>(ws.p); sa.index = P<uint32_t>(ws.index); sa.gather = P<float>(ws.gather);
    select_exact(h, sa, 1, Q, Q, R);
  }
  KC_TRY(cudaGetLastError(), "launch");
  if (R) KC_TRY(cudaMemcpyAsync(p, ws.p.p, uint64_t(Q) * R * 4, cudaMemcpyDeviceToHost, h->stream), "readback");
  KC_TRY(cudaMemcpyAsync(index, ws.index.p, Q * 4ull, cudaMemcpyDeviceToHost, h->stream), "readback");
  if (gather) KC_TRY(cudaMemcpyAsync(gather, ws.gather.p, Q * H * 4, cudaMemcpyDeviceToHost, h->stream), "readback");
  KC_TRY(cudaStreamSynchronize(h->stream), "select");
  prof_collect(h);
  return KC_OK;
}

// ---------------------------------------------------------------------------
// kc_select_noalloc: the selector over device-resident inputs with no device
// allocation. Its scratch — the two projections and the one-frame offset
// tables — is one file-scope device array, present on every GPU that loads
// this library until the process exits.
// ---------------------------------------------------------------------------
namespace {

constexpr uint32_t kNoAllocMaxQ = 256;
constexpr uint32_t kNoAllocMaxR = KC_MAX_BANK;
// layout: sq [maxQ,H] f32 | sk [maxR,H] f32 | r_off, q_off, p_off [2] u64 | query_frame [maxQ] u32
constexpr size_t kNoAllocSq = 0;
constexpr size_t kNoAllocSk = kNoAllocSq + size_t(kNoAllocMaxQ) * KC_H * 4;
constexpr size_t kNoAllocOff = kNoAllocSk + size_t(kNoAllocMaxR) * KC_H * 4;
constexpr size_t kNoAllocQf = kNoAllocOff + 6 * 8;
constexpr size_t kNoAllocBytes = kNoAllocQf + size_t(kNoAllocMaxQ) * 4;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

// Per-device address of g_noalloc_scratch (the host-side symbol is only a
// stand-in), looked up once per device.
constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices] = {};

// Writes the one-frame tables every call: every question belongs to frame 0.
__global__ void k_noalloc_tables(unsigned char* scratch, uint32_t q, uint32_t r) {
  uint64_t* off = reinterpret_cast<uint64_t*>(scratch + kNoAllocOff);
  uint32_t* qf = reinterpret_cast<uint32_t*>(scratch + kNoAllocQf);
  if (threadIdx.x == 0) {
    off[0] = 0; off[1] = r;               // r_off
    off[2] = 0; off[3] = q;               // q_off
    off[4] = 0; off[5] = uint64_t(q) * r; // p_off
  }
  for (uint32_t i = threadIdx.x; i < q; i += blockDim.x) qf[i] = 0u;
}

}  // namespace

extern "C" kc_status kc_select_noalloc(kc_handle* h, uint32_t q, uint32_t r, const float* query_output,
                                       const float* bank_keys, const float* bank_values, const float* mask,
                                       float* p, uint32_t* index, float* gather) {
  if (!h) return fail(nullptr, KC_ERR_INVALID_ARG, "handle is null");
  std::lock_guard<std::mutex> lk(h->mu);
  // no ws_epoch bump: this entry point never touches the handle's workspace,
  // so a batch resident for kc_select_batch stays usable
  DeviceGuard dg(h->device);
  if (q > kNoAllocMaxQ || r > kNoAllocMaxR) {
    char buf[160];
    snprintf(buf, sizeof buf, "kc_select_noalloc holds at most %u questions and %u bank rows (got %u, %u)",
             kNoAllocMaxQ, kNoAllocMaxR, q, r);
    return fail(h, KC_ERR_CAPACITY, buf);
  }
  if (q == 0) return KC_OK;
  if (!query_output || (r && !bank_keys) || !p || !index || (gather && r && !bank_values))
    return fail(h, KC_ERR_INVALID_ARG, "kc_select_noalloc arguments are incomplete");
  if ((reinterpret_cast<uintptr_t>(query_output) | reinterpret_cast<uintptr_t>(bank_keys)) & 15)
    return fail(h, KC_ERR_INVALID_ARG, "kc_select_noalloc: query_output and bank_keys must be 16-byte aligned");
  if (h->device < 0 || h->device >= kMaxDevices) return fail(h, KC_ERR_INVALID_ARG, "device index out of range");
  unsigned char* scratch;
  {
    std::lock_guard<std::mutex> g(g_noalloc_mu);
    if (!g_noalloc_ptr[h->device]) {
      void* ptr = nullptr;
      cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
      if (e != cudaSuccess) return cuda_fail(h, e, "kc_select_noalloc scratch address");
      g_noalloc_ptr[h->device] = ptr;
    }
    scratch = static_cast<unsigned char*>(g_noalloc_ptr[h->device]);
  }
  float* sq = reinterpret_cast<float*>(scratch + kNoAllocSq);
  float* sk = reinterpret_cast<float*>(scratch + kNoAllocSk);
  const uint64_t* off = reinterpret_cast<const uint64_t*>(scratch + kNoAllocOff);
  const uint32_t H = h->d.h;
  k_noalloc_tables<<<1, 256, 0, h->stream>>>(scratch, q, r);
  dgemm<kc::kEpiStore>(h, query_output, h->w + h->d.off_swq, sq, q, H, H);
  dgemm<kc::kEpiStore>(h, bank_keys, h->w + h->d.off_swk, sk, r, H, H);
  kc::SelectArgs sa{};
  sa.sq = sq; sa.sk = sk; sa.bank_values = bank_values;
  sa.query_frame = reinterpret_cast<const uint32_t*>(scratch + kNoAllocQf);
  sa.r_off = off; sa.q_off = off + 2; sa.p_off = off + 4;
  sa.mask = mask;
  sa.max_r = r; sa.scale = 1.0 / std::sqrt(double(H));
  sa.p = p; sa.index = index; sa.gather = gather;
  h->launches++;
  select_exact(h, sa, 1, q, q, r);
  KC_TRY(cudaGetLastError(), "kc_select_noalloc launch");
  return KC_OK;
}

static kc_status batch_host_common(kc_handle* h, const kc_batch_view* bv, DevBatch& b) {
  Workspace& ws = h->ws;
  const uint32_t F = bv->frames;
  if (!bv->rec_off || !bv->token_ids || !bv->field_roles || !bv->schema_ids || !bv->band_ids)
    return fail(h, KC_ERR_INVALID_ARG, "batch view is incomplete");
  if (bv->rec_off[0] != 0 || bv->rec_off[F] != bv->records)
    return fail(h, KC_ERR_INVALID_ARG, "rec_off must start at 0 and end at the record count");
  for (uint32_t f = 0; f < F; f++)
    if (bv->rec_off[f + 1] < bv->rec_off[f]) return fail(h, KC_ERR_INVALID_ARG, "rec_off must not decrease");
  const uint64_t N = bv->records;
  kc_status s;
  if ((s = stage(h, ws.rec_off, bv->rec_off, F + 1ull)) || (s = stage(h, ws.token_ids, bv->token_ids, N * 8)) ||
      (s = stage(h, ws.field_roles, bv->field_roles, N * 8)) || (s = stage(h, ws.schema_ids, bv->schema_ids, N)) ||
      (s = stage(h, ws.band_ids, bv->band_ids, N)))
    return s;
  b.frames = F; b.records = N; b.rec_off = P<uint64_t>(ws.rec_off);
  b.token_ids = P<uint32_t>(ws.token_ids); b.field_roles = P<uint32_t>(ws.field_roles);
  b.schema_ids = P<uint32_t>(ws.schema_ids); b.band_ids = P<uint32_t>(ws.band_ids);
  if (bv->word_ids && bv->word_alpha != 0.0f) {
    if ((s = stage(h, ws.word_ids, bv->word_ids, N * 8))) return s;
    b.word_ids = P<uint32_t>(ws.word_ids);
    b.word_alpha = bv->word_alpha;
  }
  return KC_OK;
}

}  // extern "C"

namespace {
kc_status copy_out(kc_handle* h, uint32_t frames, const kc::FrameTotals& tot, kc_batch_out* out);

// kc_forward_batch with the handle's lock held and its device current.
kc_status forward_batch_host(kc_handle* h, const kc_batch_view* bv, kc_batch_out* out) {
  if (!bv || !out || bv->frames == 0) return fail(h, KC_ERR_INVALID_ARG, "batch arguments are incomplete");
  if ((bv->schema_allow == nullptr) != (bv->band_allow == nullptr))
    return fail(h, KC_ERR_INVALID_ARG, "a mask rule needs both schema_allow and band_allow");
  if (bv->mask && bv->schema_allow)
    return fail(h, KC_ERR_INVALID_ARG, "a batch takes a mask rule or an explicit mask, not both");
  DevBatch b;
  kc_status s = batch_host_common(h, bv, b);
  if (s) return s;
  // The rule and uniforms are per batch question; their count is known only
  // after packing, so they are staged at the largest possible size.
  Workspace& ws = h->ws;
  const uint64_t N = bv->records;
  // count questions on the host to size the optional per-question arrays
  if (bv->schema_allow || bv->uniforms) {
    uint64_t nq = 0;
    for (uint64_t i = 0; i < N; i++) nq += bv->band_ids[i] == KC_QUERY_BAND;
    if (bv->schema_allow) {
      if ((s = stage(h, ws.schema_allow, bv->schema_allow, nq * 8)) || (s = stage(h, ws.band_allow, bv->band_allow, nq)))
        return s;
      b.schema_allow = P<uint32_t>(ws.schema_allow);
      b.band_allow = P<uint32_t>(ws.band_allow);
    }
    if (bv->uniforms) {
      if ((s = stage(h, ws.uniforms, bv->uniforms, nq))) return s;
      b.uniforms = P<double>(ws.uniforms);
    }
  }
  if (bv->mask) {  // sum_f Q_f * R_f, as the packer will lay p out
    uint64_t np = 0;
    for (uint32_t f = 0; f < bv->frames; f++) {
      uint64_t q = 0;
      for (uint64_t i = bv->rec_off[f]; i < bv->rec_off[f + 1]; i++) q += bv->band_ids[i] == KC_QUERY_BAND;
      np += q * (bv->rec_off[f + 1] - bv->rec_off[f] - q);
    }
    if ((s = stage(h, ws.mask, bv->mask, np))) return s;
    b.mask = P<float>(ws.mask);
    b.mask_len = np;
  }
  kc::FrameTotals tot;
  if ((s = run_batch(h, b, false, &tot))) return s;
  // the batch stays resident for kc_select_batch until ws is packed again or
  // the weights change (the last overflowed certified batch has no usable
  // tensor-core projections: its reselection runs the whole batch again)
  h->resident_epoch = h->ws_epoch;
  h->resident_precision = h->precision;
  h->resident_frames = b.frames;
  h->resident_records = b.records;
  h->resident_words = b.word_ids != nullptr;
  h->resident_alpha = b.word_alpha;
  h->resident_tot = tot;
  return copy_out(h, bv->frames, tot, out);
}

// The results of the batch in ws (p, indices, offsets, optionally the mixer's
// query output) into the caller's host buffers.
kc_status copy_out(kc_handle* h, uint32_t frames, const kc::FrameTotals& tot, kc_batch_out* out) {
  Workspace& ws = h->ws;
  out->total_p = tot.p; out->total_q = tot.q; out->total_r = tot.r; out->total_t = tot.t;
  if (tot.p > out->p_capacity || tot.q > out->q_capacity || (tot.p && !out->p) || (tot.q && !out->index))
    return fail(h, KC_ERR_CAPACITY, "output buffers are smaller than the batch's p / index");
  if (tot.p) KC_TRY(cudaMemcpyAsync(out->p, ws.p.p, tot.p * 4, cudaMemcpyDeviceToHost, h->stream), "readback");
  if (tot.q) KC_TRY(cudaMemcpyAsync(out->index, ws.index.p, tot.q * 4, cudaMemcpyDeviceToHost, h->stream), "readback");
  if (out->p_off) KC_TRY(cudaMemcpyAsync(out->p_off, ws.p_off.p, (frames + 1ull) * 8, cudaMemcpyDeviceToHost, h->stream), "readback");
  if (out->q_off) KC_TRY(cudaMemcpyAsync(out->q_off, ws.q_off.p, (frames + 1ull) * 8, cudaMemcpyDeviceToHost, h->stream), "readback");
  if (out->query_output && tot.q)
    KC_TRY(cudaMemcpyAsync(out->query_output, ws.qstate.p, tot.q * h->d.h * 4, cudaMemcpyDeviceToHost, h->stream), "readback");
  KC_TRY(wait_stream(h), "batch");
  prof_collect(h);
  return KC_OK;
}

// kc_select_batch with the handle's lock held and its device current.
kc_status select_batch_host(kc_handle* h, const kc_batch_select_view* sv, kc_batch_out* out) {
  if (!out) return fail(h, KC_ERR_INVALID_ARG, "select_batch arguments are incomplete");
  if (h->resident_epoch == 0 || h->resident_epoch != h->ws_epoch)
    return fail(h, KC_ERR_INVALID_ARG,
                "no batch is resident: run kc_forward_batch first (another call on this handle, or a weight "
                "change, since then releases it)");
  const bool rule = sv && sv->schema_allow;
  if (sv && (sv->schema_allow == nullptr) != (sv->band_allow == nullptr))
    return fail(h, KC_ERR_INVALID_ARG, "a mask rule needs both schema_allow and band_allow");
  if (rule && sv->mask) return fail(h, KC_ERR_INVALID_ARG, "a mask rule or an explicit mask, not both");
  Workspace& ws = h->ws;
  const kc::FrameTotals tot = h->resident_tot;
  DevBatch b;
  b.frames = h->resident_frames; b.records = h->resident_records; b.rec_off = P<uint64_t>(ws.rec_off);
  b.token_ids = P<uint32_t>(ws.token_ids); b.field_roles = P<uint32_t>(ws.field_roles);
  b.schema_ids = P<uint32_t>(ws.schema_ids); b.band_ids = P<uint32_t>(ws.band_ids);
  if (h->resident_words) { b.word_ids = P<uint32_t>(ws.word_ids); b.word_alpha = h->resident_alpha; }
  kc_status s;
  if (rule) {
    if ((s = stage(h, ws.schema_allow, sv->schema_allow, tot.q * 8)) || (s = stage(h, ws.band_allow, sv->band_allow, tot.q)))
      return s;
    b.schema_allow = P<uint32_t>(ws.schema_allow);
    b.band_allow = P<uint32_t>(ws.band_allow);
  }
  if (sv && sv->uniforms) {
    if ((s = stage(h, ws.uniforms, sv->uniforms, tot.q))) return s;
    b.uniforms = P<double>(ws.uniforms);
  }
  if (sv && sv->mask) {
    if ((s = stage(h, ws.mask, sv->mask, tot.p))) return s;
    b.mask = P<float>(ws.mask);
    b.mask_len = tot.p;
  }
  if (tot.q > 0) {
    const int precision = h->resident_precision;
    if (precision == KC_PRECISION_EXACT) {
      ProfScope ps(h, kStSelector);
      launch_select_exact(h, ws, b, tot, nullptr, nullptr);
      KC_TRY(cudaGetLastError(), "launch");
    } else if (h->last_overflow) {
      // the tensor-core projections overflowed the split: the batch again, whole
      kc::FrameTotals t2;
      const int saved = h->precision;
      h->precision = precision;
      s = run_batch(h, b, false, &t2);
      h->precision = saved;
      h->resident_epoch = h->ws_epoch;
      if (s) return s;
    } else {
      KC_TRY(cudaMemsetAsync(h->d_err, 0, sizeof(int), h->stream), "memset");
      KC_TRY(cudaMemsetAsync(ws.flags.p, 0, b.frames * 4ull, h->stream), "memset");
      {
        ProfScope ps(h, kStSelector);
        launch_select_fast(h, ws, b, tot);
        KC_TRY(cudaGetLastError(), "launch");
      }
      if (precision == KC_PRECISION_CERTIFIED) KC_CHECK(certify(h, ws, b, tot));
    }
  }
  return copy_out(h, b.frames, tot, out);
}
}  // namespace

extern "C" {

kc_status kc_forward_batch(kc_handle* h, const kc_batch_view* bv, kc_batch_out* out) {
  if (!h) return fail(nullptr, KC_ERR_INVALID_ARG, "handle is null");
  std::lock_guard<std::mutex> lk(h->mu);
  DeviceGuard dg(h->device);
  return forward_batch_host(h, bv, out);
}

kc_status kc_select_batch(kc_handle* h, const kc_batch_select_view* sv, kc_batch_out* out) {
  if (!h) return fail(nullptr, KC_ERR_INVALID_ARG, "handle is null");
  std::lock_guard<std::mutex> lk(h->mu);
  DeviceGuard dg(h->device);
  return select_batch_host(h, sv, out);
}

kc_status kc_forward_batch_device(kc_handle* h, const kc_batch_view* bv, kc_device_result* out) {
  if (!h) return fail(nullptr, KC_ERR_INVALID_ARG, "handle is null");
  std::lock_guard<std::mutex> lk(h->mu);
  h->ws_epoch++;  // the resident batch (kc_select_batch) is gone
  DeviceGuard dg(h->device);
  if (!bv || !out || bv->frames == 0) return fail(h, KC_ERR_INVALID_ARG, "batch arguments are incomplete");
  if (!bv->rec_off || !bv->token_ids || !bv->field_roles || !bv->schema_ids || !bv->band_ids)
    return fail(h, KC_ERR_INVALID_ARG, "batch view is incomplete");
  if ((reinterpret_cast<uintptr_t>(bv->token_ids) & 15) || (reinterpret_cast<uintptr_t>(bv->rec_off) & 7))
    return fail(h, KC_ERR_INVALID_ARG, "token_ids must be 16-byte aligned and rec_off 8-byte aligned");
  if ((bv->schema_allow == nullptr) != (bv->band_allow == nullptr))
    return fail(h, KC_ERR_INVALID_ARG, "a mask rule needs both schema_allow and band_allow");
  if (bv->mask && bv->schema_allow)
    return fail(h, KC_ERR_INVALID_ARG, "a batch takes a mask rule or an explicit mask, not both");
  DevBatch b;
  b.frames = bv->frames; b.records = bv->records; b.rec_off = bv->rec_off;
  b.token_ids = bv->token_ids; b.field_roles = bv->field_roles; b.schema_ids = bv->schema_ids;
  b.band_ids = bv->band_ids; b.schema_allow = bv->schema_allow; b.band_allow = bv->band_allow;
  b.uniforms = bv->uniforms;
  b.word_ids = bv->word_ids;
  b.word_alpha = bv->word_alpha;
  b.mask = bv->mask;
  kc::FrameTotals tot;
  kc_status s = run_batch(h, b, false, &tot);
  if (s) return s;
  out->p = P<float>(h->ws.p); out->index = P<uint32_t>(h->ws.index);
  out->p_off = P<uint64_t>(h->ws.p_off); out->q_off = P<uint64_t>(h->ws.q_off);
  out->total_p = tot.p; out->total_q = tot.q; out->total_r = tot.r; out->total_t = tot.t;
  if (h->profiling) prof_collect(h);
  return KC_OK;
}

kc_status kc_backward(kc_handle* h, const kc_frame_view* frame, const float* selection, const uint32_t* targets,
                      int has_valence, double valence, kc_backward_out* out) {
  if (!h) return fail(nullptr, KC_ERR_INVALID_ARG, "handle is null");
  std::lock_guard<std::mutex> lk(h->mu);
  h->ws_epoch++;  // the resident batch (kc_select_batch) is gone
  DeviceGuard dg(h->device);
  if (!out || !out->policy || !out->value_prediction || !out->d_selector_wq || !out->d_selector_wk ||
      !out->d_pool || !out->d_value_wv)
    return fail(h, KC_ERR_INVALID_ARG, "backward outputs are incomplete");
  DevBatch b;
  uint32_t q = 0, r = 0;
  kc_status s = stage_frame(h, frame, b, &q, &r);
  if (s) return s;
  if (q == 0) return fail(h, KC_ERR_INVALID_ARG, "the frame must contain at least one query record for the mixer");
  if (uint64_t(q) * r > out->p_capacity || q > out->q_capacity)
    return fail(h, KC_ERR_CAPACITY, "output buffers are smaller than the frame's Q/R");
  Workspace& ws = h->ws;
  BackWs& bw = h->bw;
  const double v = has_valence ? valence : std::nan("");
  if ((selection && (s = stage(h, ws.mask, selection, uint64_t(q) * r))) ||
      (targets && (s = stage(h, bw.targets, targets, q))) || (s = stage(h, bw.valence, &v, 1)))
    return s;
  kc::FrameTotals tot;
  if ((s = backward_batch(h, b, selection ? P<float>(ws.mask) : nullptr, targets ? P<uint32_t>(bw.targets) : nullptr,
                          P<double>(bw.valence), &tot, true)))
    return s;
  out->q = q;
  out->r = r;
  out->t = uint32_t(tot.t);
  if (out->d_field_states && tot.t > out->t_capacity)
    return fail(h, KC_ERR_CAPACITY, "d_field_states is smaller than the frame's active tokens");
  const uint64_t H = h->d.h;
  auto get = [&](void* dst, const DevBuf& src, uint64_t bytes) -> kc_status {
    if (bytes) KC_TRY(cudaMemcpyAsync(dst, src.p, bytes, cudaMemcpyDeviceToHost, h->stream), "readback");
    return KC_OK;
  };
  if ((s = get(out->policy, ws.p, uint64_t(q) * r * 4)) || (s = get(out->value_prediction, bw.pred, q * 4ull)) ||
      (s = get(&out->value_loss, bw.loss, 8)) || (s = get(out->d_selector_wq, bw.dswq, H * H * 4)) ||
      (s = get(out->d_selector_wk, bw.dswk, H * H * 4)) || (s = get(out->d_pool, bw.dpool, 2 * H * 4)) ||
      (s = get(out->d_value_wv, bw.dwv, 3 * H * 4)) ||
      (out->d_field_states && (s = get(out->d_field_states, bw.dfs, tot.t * H * 4))))
    return s;
  KC_TRY(cudaStreamSynchronize(h->stream), "backward");
  prof_collect(h);
  return KC_OK;
}

kc_status kc_backward_batch_device(kc_handle* h, const kc_batch_view* bv, const float* selection,
                                   const uint32_t* targets, const double* valence, kc_backward_result* out) {
  if (!h) return fail(nullptr, KC_ERR_INVALID_ARG, "handle is null");
  std::lock_guard<std::mutex> lk(h->mu);
  h->ws_epoch++;  // the resident batch (kc_select_batch) is gone
  DeviceGuard dg(h->device);
  if (!bv || !out || bv->frames == 0) return fail(h, KC_ERR_INVALID_ARG, "batch arguments are incomplete");
  if (!bv->rec_off || !bv->token_ids || !bv->field_roles || !bv->schema_ids || !bv->band_ids)
    return fail(h, KC_ERR_INVALID_ARG, "batch view is incomplete");
  if ((reinterpret_cast<uintptr_t>(bv->token_ids) & 15) || (reinterpret_cast<uintptr_t>(bv->rec_off) & 7))
    return fail(h, KC_ERR_INVALID_ARG, "token_ids must be 16-byte aligned and rec_off 8-byte aligned");
  if ((bv->schema_allow == nullptr) != (bv->band_allow == nullptr))
    return fail(h, KC_ERR_INVALID_ARG, "a mask rule needs both schema_allow and band_allow");
  DevBatch b;
  b.frames = bv->frames; b.records = bv->records; b.rec_off = bv->rec_off;
  b.token_ids = bv->token_ids; b.field_roles = bv->field_roles; b.schema_ids = bv->schema_ids;
  b.band_ids = bv->band_ids; b.schema_allow = bv->schema_allow; b.band_allow = bv->band_allow;
  kc::FrameTotals tot;
  kc_status s = backward_batch(h, b, selection, targets, valence, &tot, false);
  if (s) return s;
  BackWs& bw = h->bw;
  Workspace& ws = h->ws;
  out->policy = P<float>(ws.p); out->value_prediction = P<float>(bw.pred); out->value_loss = P<double>(bw.loss);
  out->d_selector_wq = P<float>(bw.dswq); out->d_selector_wk = P<float>(bw.dswk); out->d_pool = P<float>(bw.dpool);
  out->d_field_states = P<float>(bw.dfs); out->d_value_wv = P<float>(bw.dwv);
  out->p_off = P<uint64_t>(ws.p_off); out->q_off = P<uint64_t>(ws.q_off); out->r_off = P<uint64_t>(ws.r_off);
  out->t_off = P<uint64_t>(ws.t_off);
  out->total_p = tot.p; out->total_q = tot.q; out->total_r = tot.r; out->total_t = tot.t;
  if (h->profiling) prof_collect(h);
  return KC_OK;
}

kc_status kc_learn_frame_stats(kc_handle* h, const uint32_t* targets, double* stats) {
  if (!h) return fail(nullptr, KC_ERR_INVALID_ARG, "handle is null");
  std::lock_guard<std::mutex> lk(h->mu);
  h->ws_epoch++;  // the resident batch (kc_select_batch) is gone
  DeviceGuard dg(h->device);
  const uint32_t F = h->bw.frames;
  if (F == 0) return fail(h, KC_ERR_INVALID_ARG, "no batch has been differentiated on this handle");
  if (!stats) return fail(h, KC_ERR_INVALID_ARG, "stats is null");
  Workspace& ws = h->ws;
  kc::BatchGeo geo{P<uint32_t>(ws.query_frame), P<uint32_t>(ws.bank_frame), P<uint64_t>(ws.q_off),
                   P<uint64_t>(ws.r_off), P<uint64_t>(ws.p_off)};
  kc::k_learn_frame_stats<<<(F + 7) / 8, 256, 0, h->stream>>>(geo, P<float>(ws.p), h->bw.mask_used,
                                                              P<float>(h->bw.pred), P<double>(h->bw.loss), targets,
                                                              F, stats);
  h->launches++;
  KC_TRY(cudaGetLastError(), "learn stats");
  return KC_OK;
}

kc_status kc_learn_accumulate(kc_handle* h, const double* step, const double* value_weight, double* sums) {
  if (!h) return fail(nullptr, KC_ERR_INVALID_ARG, "handle is null");
  std::lock_guard<std::mutex> lk(h->mu);
  h->ws_epoch++;  // the resident batch (kc_select_batch) is gone
  DeviceGuard dg(h->device);
  const uint32_t F = h->bw.frames;
  if (F == 0) return fail(h, KC_ERR_INVALID_ARG, "no batch has been differentiated on this handle");
  if (!step || !value_weight || !sums) return fail(h, KC_ERR_INVALID_ARG, "learn arguments are incomplete");
  const uint64_t H = h->d.h, E = 2 * H * H + 2 * H + 3 * H;
  const uint32_t chunks = (F + kc::kLearnChunk - 1) / kc::kLearnChunk;
  KC_TRY(ensure(h, h->bw.learn_partial, uint64_t(chunks) * E * 8), "workspace");
  BackWs& bw = h->bw;
  kc::k_learn_partial<<<dim3(unsigned((E + 255) / 256), chunks), 256, 0, h->stream>>>(
      step, value_weight, P<float>(bw.dswq), P<float>(bw.dswk), P<float>(bw.dpool), P<float>(bw.dwv), F,
      P<double>(bw.learn_partial));
  kc::k_learn_sum<<<unsigned((E + 255) / 256), 256, 0, h->stream>>>(P<double>(bw.learn_partial), chunks, sums);
  h->launches += 2;
  KC_TRY(cudaGetLastError(), "learn accumulate");
  return KC_OK;
}

namespace {

bool learn_opts_ok(const kc_learn_options* o) {
  return o && o->learning_rate == o->learning_rate && o->policy_scale == o->policy_scale &&
         o->advantage_clip == o->advantage_clip && o->token_rate == o->token_rate &&
         !(o->max_parameter_abs != o->max_parameter_abs);
}

kc::LearnOpts learn_opts(const kc_learn_options* o) {
  return kc::LearnOpts{o->learning_rate, o->policy_scale, o->advantage_clip, o->max_parameter_abs, o->token_rate,
                       o->unfreeze_pool ? 1 : 0, o->unfreeze_tokens ? 1 : 0};
}

}  // namespace

kc_status kc_learn_plan(kc_handle* h, const double* rows, uint32_t frames, const kc_learn_options* o, double* step,
                        double* value_weight, double* pending, double* report) {
  if (!h) return fail(nullptr, KC_ERR_INVALID_ARG, "handle is null");
  std::lock_guard<std::mutex> lk(h->mu);
  DeviceGuard dg(h->device);
  if ((frames && (!rows || !step || !value_weight || !pending)) || !report || !learn_opts_ok(o))
    return fail(h, KC_ERR_INVALID_ARG, "learn plan arguments are incomplete");
  kc::k_learn_plan<<<1, kc::kPlanThreads, kc::kPlanSmem, h->stream>>>(rows, frames, learn_opts(o), step,
                                                                       value_weight, pending, report);
  h->launches++;
  KC_TRY(cudaGetLastError(), "learn plan");
  return KC_OK;
}

kc_status kc_learn_accumulate_rows(kc_handle* h, const uint32_t* token_ids, const uint32_t* field_roles,
                                   const double* step, const double* pending, double* row_sums, double* touched) {
  if (!h) return fail(nullptr, KC_ERR_INVALID_ARG, "handle is null");
  std::lock_guard<std::mutex> lk(h->mu);
  DeviceGuard dg(h->device);
  const uint32_t F = h->bw.frames;
  if (F == 0) return fail(h, KC_ERR_INVALID_ARG, "no batch has been differentiated on this handle");
  if (!token_ids || !field_roles || !step || !pending || !row_sums || !touched)
    return fail(h, KC_ERR_INVALID_ARG, "learn row arguments are incomplete");
  Workspace& ws = h->ws;
  uint64_t T = 0;
  KC_TRY(cudaMemcpyAsync(&T, P<uint64_t>(ws.t_off) + F, 8, cudaMemcpyDeviceToHost, h->stream), "readback");
  KC_TRY(cudaStreamSynchronize(h->stream), "learn rows");
  if (T) {
    const uint64_t warps = (T + 31) / 32;
    kc::k_learn_rows<<<unsigned((warps + 7) / 8), 256, 0, h->stream>>>(
        P<uint64_t>(ws.t_off), F, P<uint32_t>(ws.tok_recpos), token_ids, field_roles, h->token_rows, step, pending,
        P<float>(h->bw.dfs), T, h->d.token_space, row_sums, touched);
    h->launches++;
  }
  KC_TRY(cudaGetLastError(), "learn rows");
  return KC_OK;
}

kc_status kc_learn_apply(kc_handle* h, const double* sums, const double* row_sums, const double* touched,
                         const double* report, const kc_learn_options* o, double* result) {
  if (!h) return fail(nullptr, KC_ERR_INVALID_ARG, "handle is null");
  std::lock_guard<std::mutex> lk(h->mu);
  h->ws_epoch++;  // the weights may change: the resident batch (kc_select_batch) is gone
  DeviceGuard dg(h->device);
  if (!sums || !report || !result || !learn_opts_ok(o) || (o->unfreeze_tokens && (!row_sums || !touched)))
    return fail(h, KC_ERR_INVALID_ARG, "learn apply arguments are incomplete");
  const Dims& d = h->d;
  if (d.h != KC_H) return fail(h, KC_ERR_INVALID_ARG, "the device update needs the default hidden size");
  kc::LearnApplyArgs a{};
  a.page = h->w;
  a.off_swq = d.off_swq; a.off_swk = d.off_swk; a.off_val = d.off_val; a.off_pool = d.off_pool;
  a.tb_token = d.tb_token;
  a.rows = d.token_space + d.field_space;
  a.sums = sums;
  a.row_sums = o->unfreeze_tokens ? row_sums : nullptr;
  a.touched = o->unfreeze_tokens ? touched : nullptr;
  a.report = report;
  a.o = learn_opts(o);
  BackWs& bw = h->bw;
  const uint64_t elems = 2ull * d.h * d.h + 5ull * d.h + (a.row_sums ? uint64_t(a.rows) * d.h : 0);
  KC_TRY(ensure(h, bw.learn_backup, elems * 4), "workspace");
  KC_TRY(ensure(h, bw.learn_health, 4 * kc::kHealthGroups * 4), "workspace");
  KC_TRY(ensure(h, bw.learn_out, (kc::kLearnResult + kc::kLearnReport) * 8), "workspace");
  a.backup = P<float>(bw.learn_backup);
  a.health = P<unsigned>(bw.learn_health);
  a.result = P<double>(bw.learn_out);
  const unsigned grid = unsigned(std::min<uint64_t>((elems + 255) / 256, uint64_t(h->sms) * 4));
  KC_TRY(cudaMemsetAsync(a.health, 0, 4 * kc::kHealthGroups * 4, h->stream), "memset");
  kc::k_learn_health<<<grid, 256, 0, h->stream>>>(a, 0);
  kc::k_learn_backup<<<grid, 256, 0, h->stream>>>(a);
  kc::k_learn_update<<<grid, 256, 0, h->stream>>>(a);
  kc::k_learn_health<<<grid, 256, 0, h->stream>>>(a, 1);
  kc::k_learn_settle<<<grid, 256, 0, h->stream>>>(a);
  h->launches += 5;
  double out[kc::kLearnResult + kc::kLearnReport];
  KC_TRY(cudaMemcpyAsync(P<double>(bw.learn_out) + kc::kLearnResult, report, kc::kLearnReport * 8,
                         cudaMemcpyDeviceToDevice, h->stream), "copy");
  KC_TRY(cudaMemcpyAsync(out, bw.learn_out.p, sizeof out, cudaMemcpyDeviceToHost, h->stream), "readback");
  KC_TRY(cudaStreamSynchronize(h->stream), "learn apply");
  KC_TRY(cudaGetLastError(), "learn apply");
  for (int i = 0; i < kc::kLearnResult + kc::kLearnReport; i++) result[i] = out[i];
  const bool applied = out[0] != 0.0, moved = out[kc::kLearnResult + 1] != 0.0;
  if (applied && moved) {  // the selector moved: its tensor-core images and transposed copies are stale
    const size_t nf = h->mats.size() / 2, i = nf - 2;
    h->mat_max[i] = h->mat_max[nf + i] = float(out[7]);
    h->mat_max[i + 1] = h->mat_max[nf + i + 1] = float(out[8]);
    h->mat_dirty[i] = h->mat_dirty[i + 1] = h->mat_dirty[nf + i] = h->mat_dirty[nf + i + 1] = 1;
    h->oz_dirty[i] = h->oz_dirty[i + 1] = h->oz_dirty[nf + i] = h->oz_dirty[nf + i + 1] = 1;
    h->wt_sel_dirty = true;
  }
  return KC_OK;
}

kc_status kc_copy_weights(kc_handle* h, uint64_t offset, uint64_t count, float* host) {
  if (!h) return fail(nullptr, KC_ERR_INVALID_ARG, "handle is null");
  std::lock_guard<std::mutex> lk(h->mu);
  DeviceGuard dg(h->device);
  if (!host && count) return fail(h, KC_ERR_INVALID_ARG, "copy destination is null");
  if (offset > h->d.total || count > h->d.total - offset)
    return fail(h, KC_ERR_INVALID_ARG, "the range lies outside the weight page");
  if (count)
    KC_TRY(cudaMemcpyAsync(host, h->w + offset, count * 4, cudaMemcpyDeviceToHost, h->stream), "readback");
  KC_TRY(cudaStreamSynchronize(h->stream), "copy weights");
  return KC_OK;
}

kc_status kc_load_checkpoint(kc_handle* h, const void* bytes, uint64_t len, int* refusal) {
  if (!h) return fail(nullptr, KC_ERR_INVALID_ARG, "handle is null");
  std::lock_guard<std::mutex> lk(h->mu);
  h->ws_epoch++;  // the resident batch (kc_select_batch) is gone
  DeviceGuard dg(h->device);
  if (!refusal || (!bytes && len)) return fail(h, KC_ERR_INVALID_ARG, "checkpoint arguments are incomplete");
  const Dims& d = h->d;
  const unsigned char* b = static_cast<const unsigned char*>(bytes);
  auto word = [&](uint64_t i) {  // the reader copes with any alignment
    uint32_t v;
    memcpy(&v, b + 4 * i, 4);
    return v;
  };
  constexpr uint64_t kHeader = 11;
  *refusal = KC_CHECKPOINT_FITS;
  if (len < kHeader * 4) return *refusal = KC_CHECKPOINT_TRUNCATED, KC_OK;
  if (word(0) != KC_CHECKPOINT_MAGIC) return *refusal = KC_CHECKPOINT_NOT_KRYSTAL, KC_OK;
  if (word(1) > KC_CHECKPOINT_VERSION) return *refusal = KC_CHECKPOINT_LATER_FORMAT, KC_OK;
  const uint32_t geometry[7] = {d.h, d.ffn, d.enc, d.mix, d.heads, d.hd, d.route};
  for (int i = 0; i < 7; i++)
    if (word(2 + i) != geometry[i]) return *refusal = KC_CHECKPOINT_GEOMETRY, KC_OK;
  const uint64_t rows = word(9), elements = word(10);
  if (rows != h->token_rows_len) return *refusal = KC_CHECKPOINT_VOCABULARY, KC_OK;
  if (len < (kHeader + rows + elements) * 4) return *refusal = KC_CHECKPOINT_TRUNCATED, KC_OK;
  for (uint64_t i = 0; i < rows; i++)
    if (word(kHeader + i) != h->token_rows_host[i]) return *refusal = KC_CHECKPOINT_VOCABULARY, KC_OK;
  if (elements != d.total) return *refusal = KC_CHECKPOINT_GEOMETRY, KC_OK;
  const unsigned char* fl = b + (kHeader + rows) * 4;
  KC_TRY(cudaMemcpyAsync(h->w, fl, elements * 4, cudaMemcpyHostToDevice, h->stream), "checkpoint");
  // every matrix moved: largest entries for the split scales, all images stale
  auto amax = [&](uint64_t off, uint64_t n) {
    float m = 0.f;
    for (uint64_t i = 0; i < n; i++) {
      float v;
      memcpy(&v, fl + 4 * (off + i), 4);
      m = std::max(m, std::fabs(v));
    }
    return m;
  };
  const size_t nf = h->mats.size() / 2;
  for (size_t i = 0; i < nf; i++) {
    const Mat& m = h->mats[i];
    h->mat_max[i] = h->mat_max[nf + i] = amax(m.page_off, uint64_t(m.n) * m.k);
  }
  std::fill(h->mat_dirty.begin(), h->mat_dirty.end(), 1);
  std::fill(h->oz_dirty.begin(), h->oz_dirty.end(), 1);
  h->wt_blocks_dirty = h->wt_sel_dirty = true;
  KC_TRY(cudaStreamSynchronize(h->stream), "checkpoint");
  return KC_OK;
}

kc_status kc_save_checkpoint(kc_handle* h, void* out, uint64_t cap, uint64_t* written) {
  if (!h) return fail(nullptr, KC_ERR_INVALID_ARG, "handle is null");
  std::lock_guard<std::mutex> lk(h->mu);
  DeviceGuard dg(h->device);
  if (!written) return fail(h, KC_ERR_INVALID_ARG, "written is null");
  const Dims& d = h->d;
  const uint64_t rows = h->token_rows_len, bytes = (11 + rows + d.total) * 4;
  *written = bytes;
  if (cap < bytes || !out) return fail(h, KC_ERR_CAPACITY, "the checkpoint buffer is smaller than the checkpoint");
  const uint32_t header[11] = {KC_CHECKPOINT_MAGIC, KC_CHECKPOINT_VERSION, d.h, d.ffn, d.enc, d.mix, d.heads,
                               d.hd, d.route, uint32_t(rows), uint32_t(d.total)};
  unsigned char* o = static_cast<unsigned char*>(out);
  memcpy(o, header, sizeof header);
  memcpy(o + 44, h->token_rows_host.data(), rows * 4);
  KC_TRY(cudaMemcpyAsync(o + 44 + rows * 4, h->w, d.total * 4, cudaMemcpyDeviceToHost, h->stream), "checkpoint");
  KC_TRY(cudaStreamSynchronize(h->stream), "checkpoint");
  return KC_OK;
}

kc_status kc_set_precision(kc_handle* h, int mode, float tau) {
  if (!h) return fail(nullptr, KC_ERR_INVALID_ARG, "handle is null");
  std::lock_guard<std::mutex> lk(h->mu);
  if (mode != KC_PRECISION_EXACT && mode != KC_PRECISION_CERTIFIED && mode != KC_PRECISION_FAST)
    return fail(h, KC_ERR_INVALID_ARG, "unknown precision mode");
  if (tau < 0.f || !(tau == tau)) return fail(h, KC_ERR_INVALID_ARG, "tau must be a non-negative number");
  h->precision = mode;
  if (tau > 0.f) h->kappa0 = tau;
  return KC_OK;
}

kc_status kc_inject_wait_expiry(kc_handle* h, int kernel) {
  if (!h) return fail(nullptr, KC_ERR_INVALID_ARG, "handle is null");
  std::lock_guard<std::mutex> lk(h->mu);
  if (kernel != KC_INJECT_ATTN && kernel != KC_INJECT_FFN && kernel != KC_INJECT_GEMM &&
      kernel != KC_INJECT_EXACT_GEMM)
    return fail(h, KC_ERR_INVALID_ARG, "unknown tensor-core kernel for the injected expiry");
  h->inject = kernel;
  return KC_OK;
}

kc_status kc_set_stream(kc_handle* h, void* stream) {
  if (!h) return fail(nullptr, KC_ERR_INVALID_ARG, "handle is null");
  std::lock_guard<std::mutex> lk(h->mu);
  DeviceGuard dg(h->device);
  audit_collect(h);  // its readback is queued on the old stream
  const cudaStream_t next = stream ? static_cast<cudaStream_t>(stream) : h->own;
  if (next != h->stream) {
    // work on the new stream starts after everything queued on the old one
    // (the workspace, and buffers retired but not yet freed, are shared)
    cudaEvent_t ev;
    KC_TRY(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming), "event");
    cudaError_t e = cudaEventRecord(ev, h->stream);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(next, ev, 0);
    cudaEventDestroy(ev);
    KC_TRY(e, "stream order");
  }
  h->stream = next;
  return KC_OK;
}

void* kc_get_stream(kc_handle* h) { return h ? static_cast<void*>(h->stream) : nullptr; }

kc_status kc_synchronize(kc_handle* h) {
  if (!h) return fail(nullptr, KC_ERR_INVALID_ARG, "handle is null");
  DeviceGuard dg(h->device);
  cudaError_t e = cudaStreamSynchronize(h->stream);
  if (e != cudaSuccess) return cuda_fail(h, e, "synchronize");
  return KC_OK;
}

kc_status kc_profile(kc_handle* h, int enable) {
  if (!h) return fail(nullptr, KC_ERR_INVALID_ARG, "handle is null");
  std::lock_guard<std::mutex> lk(h->mu);
  h->profiling = enable != 0;
  return KC_OK;
}

kc_status kc_profile_read(kc_handle* h, kc_stage_times* out, int reset) {
  if (!h || !out) return fail(h, KC_ERR_INVALID_ARG, "arguments are null");
  std::lock_guard<std::mutex> lk(h->mu);
  DeviceGuard dg(h->device);
  prof_collect(h);
  audit_collect(h);
  unsigned long long listed = 0;
  if (h->d_oz_word) {
    cudaMemcpyAsync(&listed, h->d_oz_word + 2, sizeof listed, cudaMemcpyDeviceToHost, h->stream);
    cudaStreamSynchronize(h->stream);
    if (reset) cudaMemsetAsync(h->d_oz_word + 2, 0, sizeof listed, h->stream);
  }
  *out = h->prof;
  out->launches = h->launches;
  out->cert_kappa0 = double(h->kappa0) * h->kappa_mul;
  out->oz_listed = listed;
  if (reset) h->prof = kc_stage_times{};
  return KC_OK;
}

uint64_t kc_launch_count(kc_handle* h) { return h ? h->launches : 0; }

void kc_destroy(kc_handle* h) {
  if (!h) return;
  {
    std::lock_guard<std::mutex> lk(h->mu);
    DeviceGuard dg(h->device);
    if (h->own) cudaStreamSynchronize(h->own);
    cudaStreamSynchronize(h->stream);
    release_retired(h);
    DevBuf* bufs[] = {&h->ws.rec_off, &h->ws.token_ids, &h->ws.field_roles, &h->ws.schema_ids, &h->ws.band_ids,
                      &h->ws.schema_allow, &h->ws.band_allow, &h->ws.uniforms, &h->ws.mask, &h->ws.bank_schema,
                      &h->ws.bank_band, &h->ws.rec_meta, &h->ws.frame_t, &h->ws.frame_q, &h->ws.frame_r,
                      &h->ws.t_off, &h->ws.q_off, &h->ws.r_off, &h->ws.p_off, &h->ws.totals, &h->ws.tok_recpos,
                      &h->ws.rec_start, &h->ws.rec_row, &h->ws.bank_rec, &h->ws.bank_frame, &h->ws.query_rec,
                      &h->ws.query_frame, &h->ws.x, &h->ws.qkv, &h->ws.bk, &h->ws.bv, &h->ws.mk, &h->ws.mv,
                      &h->ws.qstate, &h->ws.mq, &h->ws.mh, &h->ws.sq, &h->ws.sk, &h->ws.p, &h->ws.index,
                      &h->ws.gather, &h->ws.rows_val, &h->ws.rows_off, &h->ws.word_ids, &h->ws_fb.word_ids,
                      &h->ws.tile_row, &h->ws.row_rc};
    for (DevBuf* b : bufs)
      if (b->p) cudaFree(b->p), b->p = nullptr;
    Workspace& f = h->ws_fb;
    DevBuf* fbufs[] = {&f.rec_off, &f.token_ids, &f.field_roles, &f.schema_ids, &f.band_ids, &f.schema_allow,
                       &f.band_allow, &f.uniforms, &f.mask, &f.bank_schema, &f.bank_band, &f.rec_meta, &f.frame_t,
                       &f.frame_q, &f.frame_r, &f.t_off, &f.q_off, &f.r_off, &f.p_off, &f.totals, &f.tok_recpos,
                       &f.rec_start, &f.rec_row, &f.bank_rec, &f.bank_frame, &f.query_rec, &f.query_frame, &f.x,
                       &f.qkv, &f.bk, &f.bv, &f.mk, &f.mv, &f.qstate, &f.mq, &f.mh, &f.sq, &f.sk, &f.p, &f.index,
                       &f.gather, &f.rows_val, &f.rows_off, &f.flags, &f.list, &h->ws.flags, &h->ws.list,
                       &h->images};
    for (DevBuf* b : fbufs)
      if (b->p) cudaFree(b->p), b->p = nullptr;
    BackWs& k = h->bw;
    DevBuf* bbufs[] = {&k.mask, &k.targets, &k.valence, &k.enc_qkv, &k.enc_p, &k.enc_h1, &k.mix_q, &k.mix_k,
                       &k.mix_v, &k.mix_p, &k.mix_h1, &k.gather, &k.offered, &k.n_allowed, &k.pred, &k.dpred,
                       &k.loss, &k.dwv, &k.dquery, &k.dig, &k.dag, &k.dscore, &k.dqp, &k.dkp, &k.dbk, &k.dbv,
                       &k.dswq, &k.dswk, &k.dh1, &k.ads, &k.mdq, &k.mdk, &k.mdv, &k.tok_ds, &k.dfs, &k.dpool,
                       &k.edqkv, &k.learn_partial, &h->wt};
    for (DevBuf* b : bbufs)
      if (b->p) cudaFree(b->p), b->p = nullptr;
    if (h->d_err) cudaFree(h->d_err);
    if (h->d_oz_word) cudaFree(h->d_oz_word);
    if (h->h_oz_err) cudaFreeHost(h->h_oz_err);
    if (h->h_err) cudaFreeHost(h->h_err);
    if (h->d_audit) cudaFree(h->d_audit);
    if (h->h_audit) cudaFreeHost(h->h_audit);
    if (h->h_flags_pinned) cudaFreeHost(h->h_flags_pinned);
    for (auto& pr : h->ev_pool) {
      cudaEventDestroy(pr.first);
      cudaEventDestroy(pr.second);
    }
    if (h->w) cudaFree(h->w);
    if (h->token_rows) cudaFree(h->token_rows);
    if (h->h_tot) cudaFreeHost(h->h_tot);
    if (h->own) cudaStreamDestroy(h->own);
  }
  const int dev = h->device;
  DeviceGuard dg(dev);  // buffers not listed above free themselves here, with their device current
  delete h;
}

const char* kc_last_error(kc_handle* h) { return h ? h->err.c_str() : g_create_error.c_str(); }

}  // extern "C"

#include "stream.cuh"
