// krystal_oracle.cpp — CPU restatement of Krystal's frame forward + selector.
//
// TEST INFRASTRUCTURE ONLY (the checker; never linked by the product).
// Each function cites the reference TypeScript it follows, by file:line
// within the reference project (packages/...). The JavaScript numeric model
// is kept: f64 arithmetic, f32 rounding at each Float32Array store, the same
// loop orders. Build with -ffp-contract=off (see Makefile).
#include "krystal_oracle.h"

#include <cmath>
#include <cstdint>
#include <cstring>
#include <atomic>
#include <thread>
#include <vector>

namespace {

constexpr uint32_t kRecordWidth = 8;     // BRAIN_LIMITS.recordWidth (schema krystal-engine-schema.ts:97)
constexpr uint32_t kPadToken = 0;        // KRYSTAL_SENTINEL_TOKENS.pad (:56)
constexpr uint32_t kQueryBand = 5;       // index of "query" in BRAIN_FRAME_BANDS (:150-172)
constexpr uint32_t kStreamQuery = 1;     // STREAM_QUERY (model.ts:269)
constexpr uint32_t kInvalidU32 = 0xffffffffu;
constexpr float kNegInf = -1e30f;        // NEG_INF (oracle.ts:36), as stored in a Float32Array

// Math.max(a, b): NaN if either is NaN; +0 beats -0.
inline double js_max(double a, double b) {
  if (a != a || b != b) return NAN;
  if (a == b) return std::signbit(a) ? b : a;
  return a > b ? a : b;
}

inline float f32(double v) { return static_cast<float>(v); }

struct Layout {
  uint64_t emb, enc, pool, mixer, sel_wq, sel_wk, decision, value, total;
  uint64_t block;  // floats per encoder/mixer block
  // table bases inside the embeddings page (model.ts:102-124)
  uint64_t tb_token, tb_field, tb_schema, tb_band, tb_stream, tb_pos;
};

Layout layout_of(const ko_dims* d) {
  Layout L{};
  const uint64_t h = d->hidden, f = d->ffn;
  uint64_t cursor = 0;
  L.tb_token = cursor; cursor += uint64_t(d->token_space) * h;
  L.tb_field = cursor; cursor += uint64_t(d->field_space) * h;
  L.tb_schema = cursor; cursor += uint64_t(d->schema_space) * h;
  L.tb_band = cursor; cursor += uint64_t(d->band_space) * h;
  L.tb_stream = cursor; cursor += uint64_t(d->stream_space) * h;
  L.tb_pos = cursor; cursor += uint64_t(d->pos_space) * h;
  L.emb = 0;
  L.block = 3 * h * h + 2 * f * h;
  L.enc = cursor; cursor += L.block * d->enc_blocks;
  L.pool = cursor; cursor += 2 * h;
  L.mixer = cursor; cursor += L.block * d->mixer_blocks;
  L.sel_wq = cursor; cursor += h * h;
  L.sel_wk = cursor; cursor += h * h;
  L.decision = cursor; cursor += uint64_t(d->route_kinds) * 3 * h;
  L.value = cursor; cursor += 3 * h;
  L.total = cursor;
  return L;
}

// mulberry32 (model.ts:186-195). Math.imul is the low 32 bits of the product;
// `(t + imul(..)) ^ t` wraps through ToInt32, i.e. a uint32 add.
struct Mulberry32 {
  uint32_t a;
  explicit Mulberry32(uint32_t seed) : a(seed) {}
  double next() {
    a = a + 0x6d2b79f5u;
    uint32_t t = (a ^ (a >> 15)) * (1u | a);
    t = (t + ((t ^ (t >> 7)) * (61u | t))) ^ t;
    return double(t ^ (t >> 14)) / 4294967296.0;
  }
};

// xavierUniform (model.ts:197-202)
void xavier_uniform(uint64_t out, uint64_t in, Mulberry32& rand, float* dst) {
  const double limit = std::sqrt(6.0 / double(out + in));
  for (uint64_t i = 0; i < out * in; i++) dst[i] = f32((rand.next() * 2 - 1) * limit);
}

// normalTable (model.ts:204-215): Box–Muller, two values per pair of draws.
void normal_table(uint64_t n, Mulberry32& rand, double std_, float* dst) {
  const double two_pi = 2 * M_PI;
  for (uint64_t i = 0; i < n; i += 2) {
    const double u1 = js_max(rand.next(), 1e-12);
    const double u2 = rand.next();
    const double r = std::sqrt(-2 * std::log(u1));
    dst[i] = f32(r * std::cos(two_pi * u2) * std_);
    if (i + 1 < n) dst[i + 1] = f32(r * std::sin(two_pi * u2) * std_);
  }
}

// softmaxRow (oracle.ts:38-49): max over the stored f32 values; each exp is
// stored f32 while the running sum keeps the unrounded f64 value.
void softmax_row(float* v, uint32_t count) {
  double mx = -INFINITY;
  for (uint32_t i = 0; i < count; i++) mx = js_max(mx, v[i]);
  double sum = 0;
  for (uint32_t i = 0; i < count; i++) {
    const double e = std::exp(double(v[i]) - mx);
    v[i] = f32(e);
    sum += e;
  }
  const double inv = 1 / js_max(sum, 1e-20);
  for (uint32_t i = 0; i < count; i++) v[i] = f32(double(v[i]) * inv);
}

// matmulOracle (oracle.ts:114-125): y[m,o] = Σ_d x[m,d]·w[o,d], f64 in d order.
void matmul(const float* x, const float* w, uint64_t rows, uint32_t out_dim, uint32_t in_dim, float* y) {
  for (uint64_t m = 0; m < rows; m++) {
    const float* xr = x + m * in_dim;
    for (uint32_t o = 0; o < out_dim; o++) {
      const float* wr = w + uint64_t(o) * in_dim;
      double value = 0;
      for (uint32_t d = 0; d < in_dim; d++) value += double(xr[d]) * double(wr[d]);
      y[m * out_dim + o] = f32(value);
    }
  }
}

// reluOracle (oracle.ts:107-111): Math.max(0, v).
void relu_inplace(float* v, uint64_t n) {
  for (uint64_t i = 0; i < n; i++) v[i] = f32(js_max(0.0, v[i]));
}

// addInPlace (oracle.ts:137-139)
void add_inplace(float* a, const float* b, uint64_t n) {
  for (uint64_t i = 0; i < n; i++) a[i] = f32(double(a[i]) + double(b[i]));
}

// attentionOracle (oracle.ts:64-105). `local_start/local_count` restrict each
// query row to its record's key range (the encoder); NULL means all kRows.
// In local mode a record mask may carry the same-word bias (compileRecordMask,
// masks.ts:167-198): `words` holds each compact token's word id, and two
// tokens of one record with the same valid id get the f32 `alpha` as their
// mask entry (every other in-record entry is 0).
void attention(const float* q, const float* k, const float* v, const float* mask, uint64_t q_rows, uint64_t k_rows,
               uint32_t h, uint32_t heads, uint32_t head_dim, const uint32_t* local_start,
               const uint32_t* local_count, float* out, const uint32_t* words = nullptr, float alpha = 0.0f) {
  std::vector<float> scores(k_rows ? k_rows : 1);
  const double scale = 1 / std::sqrt(double(head_dim));
  for (uint64_t i = 0; i < q_rows * h; i++) out[i] = 0;
  for (uint32_t head = 0; head < heads; head++) {
    const uint32_t hb = head * head_dim;
    for (uint64_t i = 0; i < q_rows; i++) {
      const uint64_t from = local_start ? local_start[i] : 0;
      const uint64_t to = local_start ? from + local_count[i] : k_rows;
      for (uint64_t j = from; j < to; j++) {
        double s = 0;
        for (uint32_t dd = 0; dd < head_dim; dd++) s += double(q[i * h + hb + dd]) * double(k[j * h + hb + dd]);
        double m = mask ? double(mask[i * k_rows + j]) : 0.0;
        if (words && alpha != 0.0f && words[i] != kInvalidU32 && words[i] == words[j]) m = double(alpha);
        scores[j] = f32(s * scale + m);
      }
      bool all_blocked = true;
      for (uint64_t j = from; j < to; j++)
        if (scores[j] >= -1e29) { all_blocked = false; break; }
      if (all_blocked) {
        for (uint64_t j = from; j < to; j++) scores[j] = 0;
      } else {
        softmax_row(scores.data() + from, uint32_t(to - from));
      }
      for (uint32_t dd = 0; dd < head_dim; dd++) {
        double value = 0;
        for (uint64_t j = from; j < to; j++) value += double(scores[j]) * double(v[j * h + hb + dd]);
        out[i * h + hb + dd] = f32(value);
      }
    }
  }
}

// ffnOracle (oracle.ts:127-135)
void ffn(const float* x, const float* w1, const float* w2, uint64_t rows, uint32_t h, uint32_t f, float* hidden,
         float* out) {
  matmul(x, w1, rows, f, h, hidden);
  relu_inplace(hidden, rows * f);
  matmul(hidden, w2, rows, h, f, out);
}

// poolRecord (oracle.ts:186-224)
void pool_record(const float* states, uint32_t start, uint32_t count, const float* pool, uint32_t h, float* key,
                 float* value) {
  for (uint32_t d = 0; d < h; d++) key[d] = value[d] = 0;
  if (count == 0) return;
  const double scale = 1 / std::sqrt(double(h));
  float ks_[kRecordWidth], vs_[kRecordWidth];
  std::vector<float> ksv, vsv;
  float* ks = ks_;
  float* vs = vs_;
  if (count > kRecordWidth) {
    ksv.resize(count); vsv.resize(count);
    ks = ksv.data(); vs = vsv.data();
  }
  for (uint32_t j = 0; j < count; j++) {
    double a = 0, b = 0;
    for (uint32_t d = 0; d < h; d++) {
      const double s = states[uint64_t(start + j) * h + d];
      a += double(pool[d]) * s;
      b += double(pool[h + d]) * s;
    }
    ks[j] = f32(a * scale);
    vs[j] = f32(b * scale);
  }
  softmax_row(ks, count);
  softmax_row(vs, count);
  for (uint32_t d = 0; d < h; d++) {
    double ka = 0, va = 0;
    for (uint32_t j = 0; j < count; j++) {
      const double s = states[uint64_t(start + j) * h + d];
      ka += double(ks[j]) * s;
      va += double(vs[j]) * s;
    }
    key[d] = f32(ka);
    value[d] = f32(va);
  }
}

struct Active {
  std::vector<uint32_t> tokens, offset, count, stream, records, bank, query;
};

// compileActiveFrame (masks.ts:65-101)
void compile_active(uint32_t slots, const uint32_t* token_ids, const uint32_t* band_ids, const uint32_t* active_idx,
                    Active& a) {
  a.tokens.clear(); a.records.clear(); a.bank.clear(); a.query.clear();
  a.offset.assign(slots, kInvalidU32);
  a.count.assign(slots, 0);
  a.stream.assign(slots, 0);
  for (uint32_t i = 0; i < slots; i++) {
    const uint32_t slot = active_idx ? active_idx[i] : i;
    if (slot == kInvalidU32 || slot >= slots) break;  // unoccupied tail
    a.records.push_back(slot);
    a.offset[slot] = uint32_t(a.tokens.size());
    uint32_t c = 0;
    for (uint32_t local = 0; local < kRecordWidth; local++) {
      const uint32_t ft = slot * kRecordWidth + local;
      if (token_ids[ft] != kPadToken) { a.tokens.push_back(ft); c++; }
    }
    a.count[slot] = c;
    a.stream[slot] = band_ids[slot] == kQueryBand ? kStreamQuery : 0;
  }
  for (uint32_t slot : a.records) (a.stream[slot] != kStreamQuery ? a.bank : a.query).push_back(slot);
}

// selectorOracle (oracle.ts:332-382) and sampleRow (sampling.ts:41-57).
int32_t sample_row(const float* p, uint32_t count, double uniform) {
  double cumulative = 0;
  int32_t last = -1;
  for (uint32_t j = 0; j < count; j++) {
    const double w = p[j];
    if (!(w > 0)) continue;
    last = int32_t(j);
    cumulative += w;
    if (uniform < cumulative) return int32_t(j);
  }
  return last;
}

void selector(const float* query, const float* bank_keys, const float* bank_values, const float* mask,
              const float* wq, const float* wk, uint32_t q, uint32_t r, uint32_t h, const double* uniforms,
              float* p, float* gather, uint32_t* index) {
  std::vector<float> qp(uint64_t(q) * h), kp(uint64_t(r) * h), scores(r ? r : 1);
  matmul(query, wq, q, h, h, qp.data());
  matmul(bank_keys, wk, r, h, h, kp.data());
  const double scale = 1 / std::sqrt(double(h));
  for (uint32_t i = 0; i < q; i++) {
    for (uint32_t j = 0; j < r; j++) {
      double s = 0;
      for (uint32_t d = 0; d < h; d++) s += double(qp[uint64_t(i) * h + d]) * double(kp[uint64_t(j) * h + d]);
      scores[j] = f32(s * scale + double(mask ? mask[uint64_t(i) * r + j] : 0.0f));
    }
    bool all_blocked = true;  // scores.every(score => score < -1e29)
    for (uint32_t j = 0; j < r; j++)
      if (!(scores[j] < -1e29)) { all_blocked = false; break; }
    if (all_blocked) {
      for (uint32_t j = 0; j < r; j++) scores[j] = 0;
    } else {
      softmax_row(scores.data(), r);
    }
    uint32_t best = 0;
    for (uint32_t j = 0; j < r; j++) {
      p[uint64_t(i) * r + j] = scores[j];
      if (scores[j] > scores[best]) best = j;
    }
    if (all_blocked) {
      index[i] = kInvalidU32;
    } else if (uniforms) {
      const int32_t drawn = sample_row(p + uint64_t(i) * r, r, uniforms[i]);
      index[i] = drawn < 0 ? kInvalidU32 : uint32_t(drawn);
    } else {
      index[i] = best;
    }
    if (gather) {
      for (uint32_t d = 0; d < h; d++) {
        double g = 0;
        for (uint32_t j = 0; j < r; j++) g += double(scores[j]) * double(bank_values[uint64_t(j) * h + d]);
        gather[uint64_t(i) * h + d] = f32(g);
      }
    }
  }
}

// brainForwardOracle (oracle.ts:231-299), with fieldEmbed (:151-184) inline.
// Returns -1 if a token or role id has no row in token_rows, or a row or a
// schema/band id falls outside its table (the reference reads `undefined`).
int forward(const ko_dims* d, const float* W, const uint32_t* token_rows, uint32_t token_rows_len, uint32_t slots,
            const uint32_t* token_ids, const uint32_t* field_roles, const uint32_t* schema_ids,
            const uint32_t* band_ids, const Active& a, const float* mixer_mask, float* field_states,
            float* bank_keys, float* bank_values, float* query_keys, float* query_values_premix,
            float* query_output, const uint32_t* word_ids = nullptr, float alpha = 0.0f) {
  const Layout L = layout_of(d);
  const uint32_t h = d->hidden, f = d->ffn;
  const uint64_t t = a.tokens.size();
  const uint32_t r = uint32_t(a.bank.size()), q = uint32_t(a.query.size());
  (void)slots;

  // recordRanges (masks.ts:120-133)
  std::vector<uint32_t> rs(t), rc(t);
  for (uint32_t slot : a.records)
    for (uint32_t i = a.offset[slot]; i < a.offset[slot] + a.count[slot]; i++) { rs[i] = a.offset[slot]; rc[i] = a.count[slot]; }

  // 1. fieldEmbed: six rows summed in order, stored f32.
  std::vector<float> x(t * h);
  const float* table = W + L.emb;
  for (uint64_t ti = 0; ti < t; ti++) {
    const uint32_t ft = a.tokens[ti];
    const uint32_t slot = ft >> 3, local = ft & 7;
    const uint32_t tid = token_ids[ft], rid = field_roles[ft];
    if (tid >= token_rows_len || rid >= token_rows_len) return -1;
    const uint32_t tok = token_rows[tid], role = token_rows[rid];
    const uint32_t schema = schema_ids[slot], band = band_ids[slot], stream = a.stream[slot];
    if (tok >= d->token_space || role >= d->field_space || schema >= d->schema_space || band >= d->band_space ||
        local >= d->pos_space)
      return -1;
    for (uint32_t dd = 0; dd < h; dd++) {
      double value = 0;
      value += table[L.tb_token + uint64_t(tok) * h + dd];
      value += table[L.tb_field + uint64_t(role) * h + dd];
      value += table[L.tb_schema + uint64_t(schema) * h + dd];
      value += table[L.tb_band + uint64_t(band) * h + dd];
      value += table[L.tb_stream + uint64_t(stream) * h + dd];
      value += table[L.tb_pos + uint64_t(local) * h + dd];
      x[ti * h + dd] = f32(value);
    }
  }

  // the same-word bias's labels per compact token (indexed like activeTokens)
  std::vector<uint32_t> words;
  if (word_ids && alpha != 0.0f) {
    words.resize(t);
    for (uint64_t ti = 0; ti < t; ti++) words[ti] = word_ids[a.tokens[ti]];
  }

  // 2. Encoder blocks.
  std::vector<float> qb(t * h), kb(t * h), vb(t * h), attn(t * h), hid(t * f), ff(t * h);
  for (uint32_t b = 0; b < d->enc_blocks; b++) {
    const float* blk = W + L.enc + L.block * b;
    const float *wq = blk, *wk = blk + h * h, *wv = blk + 2 * h * h, *w1 = blk + 3 * h * h,
                *w2 = blk + 3 * h * h + uint64_t(f) * h;
    matmul(x.data(), wq, t, h, h, qb.data());
    matmul(x.data(), wk, t, h, h, kb.data());
    matmul(x.data(), wv, t, h, h, vb.data());
    attention(qb.data(), kb.data(), vb.data(), nullptr, t, t, h, d->heads, d->head_dim, rs.data(), rc.data(),
              attn.data(), words.empty() ? nullptr : words.data(), alpha);
    add_inplace(x.data(), attn.data(), t * h);
    ffn(x.data(), w1, w2, t, h, f, hid.data(), ff.data());
    add_inplace(x.data(), ff.data(), t * h);
  }
  if (field_states) std::memcpy(field_states, x.data(), t * h * sizeof(float));

  // 3. Pooling.
  const float* pool = W + L.pool;
  std::vector<float> qk(uint64_t(q) * h), qv(uint64_t(q) * h);
  for (uint32_t i = 0; i < r; i++) {
    const uint32_t slot = a.bank[i];
    pool_record(x.data(), a.offset[slot], a.count[slot], pool, h, bank_keys + uint64_t(i) * h,
                bank_values + uint64_t(i) * h);
  }
  for (uint32_t i = 0; i < q; i++) {
    const uint32_t slot = a.query[i];
    pool_record(x.data(), a.offset[slot], a.count[slot], pool, h, qk.data() + uint64_t(i) * h,
                qv.data() + uint64_t(i) * h);
  }
  if (query_keys) std::memcpy(query_keys, qk.data(), qk.size() * sizeof(float));
  if (query_values_premix) std::memcpy(query_values_premix, qv.data(), qv.size() * sizeof(float));

  // 4. Mixer blocks: the query state starts as the pooled query values.
  std::vector<float>& query = qv;
  std::vector<float> mq(uint64_t(q) * h), mk(uint64_t(r) * h), mv(uint64_t(r) * h), mattn(uint64_t(q) * h),
      mhid(uint64_t(q) * f), mff(uint64_t(q) * h);
  std::vector<float> zeros;
  const float* mmask = mixer_mask;
  if (!mmask) { zeros.assign(uint64_t(q) * r + 1, 0.0f); mmask = zeros.data(); }
  for (uint32_t b = 0; b < d->mixer_blocks; b++) {
    const float* blk = W + L.mixer + L.block * b;
    const float *wq = blk, *wk = blk + h * h, *wv = blk + 2 * h * h, *w1 = blk + 3 * h * h,
                *w2 = blk + 3 * h * h + uint64_t(f) * h;
    matmul(query.data(), wq, q, h, h, mq.data());
    matmul(bank_keys, wk, r, h, h, mk.data());
    matmul(bank_values, wv, r, h, h, mv.data());
    attention(mq.data(), mk.data(), mv.data(), mmask, q, r, h, d->heads, d->head_dim, nullptr, nullptr, mattn.data());
    add_inplace(query.data(), mattn.data(), uint64_t(q) * h);
    ffn(query.data(), w1, w2, q, h, f, mhid.data(), mff.data());
    add_inplace(query.data(), mff.data(), uint64_t(q) * h);
  }
  std::memcpy(query_output, query.data(), query.size() * sizeof(float));
  return 0;
}

// ---------------------------------------------------------------------------
// Backward (packages/krystal/src/forward/backward.ts), as host/gradients.ts:
// 30-66 runs it for a session: context "available", the argument slot given
// nothing to aim at (it contributes exactly zero), no route-kind labels.
// ---------------------------------------------------------------------------

// attentionWithP (backward.ts:580-618) with p kept per query row over its key
// window: p_row[(head*q_rows + i) * kw + (j - from)], kw = window width.
void attention_with_p(const float* q, const float* k, const float* v, const float* mask, uint64_t q_rows,
                      uint64_t k_rows, uint32_t h, uint32_t heads, uint32_t head_dim, const uint32_t* local_start,
                      const uint32_t* local_count, uint32_t kw, float* out, float* p) {
  std::vector<float> scores(k_rows ? k_rows : 1);
  const double scale = 1 / std::sqrt(double(head_dim));
  for (uint64_t i = 0; i < q_rows * h; i++) out[i] = 0;
  for (uint32_t head = 0; head < heads; head++) {
    const uint32_t hb = head * head_dim;
    for (uint64_t i = 0; i < q_rows; i++) {
      const uint64_t from = local_start ? local_start[i] : 0;
      const uint64_t to = local_start ? from + local_count[i] : k_rows;
      for (uint64_t j = from; j < to; j++) {
        double s = 0;
        for (uint32_t dd = 0; dd < head_dim; dd++) s += double(q[i * h + hb + dd]) * double(k[j * h + hb + dd]);
        scores[j] = f32(s * scale + (mask ? double(mask[i * k_rows + j]) : 0.0));
      }
      bool all_blocked = true;
      for (uint64_t j = from; j < to; j++)
        if (scores[j] >= -1e29) { all_blocked = false; break; }
      if (all_blocked) {
        for (uint64_t j = from; j < to; j++) scores[j] = 0;
      } else {
        softmax_row(scores.data() + from, uint32_t(to - from));
      }
      for (uint64_t j = from; j < to; j++) p[(uint64_t(head) * q_rows + i) * kw + (j - from)] = scores[j];
      for (uint32_t dd = 0; dd < head_dim; dd++) {
        double value = 0;
        for (uint64_t j = from; j < to; j++) value += double(scores[j]) * double(v[j * h + hb + dd]);
        out[i * h + hb + dd] = f32(value);
      }
    }
  }
}

// attentionBackwardScores (backward.ts:79-115) then attentionBackwardQkv
// (:117-166) for one attention, p in the windowed layout above. For the
// dense (mixer) case the window is the whole key range (kw = k_rows).
void attention_backward(const float* d_out, const float* q, const float* k, const float* v, const float* p,
                        uint64_t q_rows, uint64_t k_rows, uint32_t h, uint32_t heads, uint32_t head_dim,
                        const uint32_t* local_start, const uint32_t* local_count, uint32_t kw, float* dq, float* dk,
                        float* dv) {
  std::vector<float> d_scores(uint64_t(heads) * q_rows * kw + 1, 0.0f), dp(k_rows ? k_rows : 1);
  for (uint32_t head = 0; head < heads; head++) {
    for (uint64_t i = 0; i < q_rows; i++) {
      const uint64_t from = local_start ? local_start[i] : 0;
      const uint64_t to = local_start ? from + local_count[i] : k_rows;
      const float* prow = p + (uint64_t(head) * q_rows + i) * kw;
      double row_sum = 0;
      for (uint64_t j = from; j < to; j++) {
        double s = 0;
        for (uint32_t d = 0; d < head_dim; d++)
          s += double(d_out[i * h + head * head_dim + d]) * double(v[j * h + head * head_dim + d]);
        dp[j] = f32(s);
        row_sum += double(prow[j - from]) * s;
      }
      for (uint64_t j = from; j < to; j++)
        d_scores[(uint64_t(head) * q_rows + i) * kw + (j - from)] = f32(double(prow[j - from]) * (double(dp[j]) - row_sum));
    }
  }
  const double scale = 1 / std::sqrt(double(head_dim));
  for (uint64_t i = 0; i < q_rows; i++) {
    const uint64_t from = local_start ? local_start[i] : 0;
    const uint64_t to = local_start ? from + local_count[i] : k_rows;
    for (uint32_t col = 0; col < h; col++) {
      const uint32_t head = col / head_dim;
      double acc = 0;
      for (uint64_t j = from; j < to; j++)
        acc += double(d_scores[(uint64_t(head) * q_rows + i) * kw + (j - from)]) * double(k[j * h + col]);
      dq[i * h + col] = f32(acc * scale);
    }
  }
  // keys read the same windows the other way round: for the local case a key
  // j is scored by its own record's rows; kw-relative index of j in row i's
  // window is j - start[i]
  for (uint64_t j = 0; j < k_rows; j++) {
    const uint64_t from = local_start ? local_start[j] : 0;
    const uint64_t to = local_start ? from + local_count[j] : q_rows;
    for (uint32_t col = 0; col < h; col++) {
      const uint32_t head = col / head_dim;
      double acc_k = 0, acc_v = 0;
      for (uint64_t i = from; i < to; i++) {
        const uint64_t wi = local_start ? j - local_start[i] : j;
        acc_k += double(d_scores[(uint64_t(head) * q_rows + i) * kw + wi]) * double(q[i * h + col]);
        acc_v += double(p[(uint64_t(head) * q_rows + i) * kw + wi]) * double(d_out[i * h + col]);
      }
      dk[j * h + col] = f32(acc_k * scale);
      dv[j * h + col] = f32(acc_v);
    }
  }
}

// matmulBackInput (backward.ts:548-557): dX[m,k] = sum_n dY[m,n] W[n,k]
void matmul_back_input(const float* dy, const float* w, uint64_t m, uint32_t n, uint32_t k, float* dx) {
  for (uint64_t i = 0; i < m; i++)
    for (uint32_t j = 0; j < k; j++) {
      double s = 0;
      for (uint32_t l = 0; l < n; l++) s += double(dy[i * n + l]) * double(w[uint64_t(l) * k + j]);
      dx[i * k + j] = f32(s);
    }
}

// matmulBackWeight (backward.ts:560-569): dW[n,k] = sum_m dY[m,n] X[m,k]
void matmul_back_weight(const float* dy, const float* x, uint64_t m, uint32_t n, uint32_t k, float* dw) {
  for (uint32_t i = 0; i < n; i++)
    for (uint32_t j = 0; j < k; j++) {
      double s = 0;
      for (uint64_t l = 0; l < m; l++) s += double(dy[l * n + i]) * double(x[l * k + j]);
      dw[uint64_t(i) * k + j] = f32(s);
    }
}

// poolBackward (backward.ts:184-262) over the records listed, accumulating
// into d_states (f32 store per add) and d_pool (f32 store per add).
void pool_backward(const float* states, const std::vector<uint32_t>& recs, const Active& a, const float* pool,
                   const float* d_keys, const float* d_values, uint32_t h, float* d_states, float* d_pool) {
  const double scale = 1 / std::sqrt(double(h));
  for (size_t rec = 0; rec < recs.size(); rec++) {
    const uint32_t slot = recs[rec];
    const uint32_t start = a.offset[slot], count = a.count[slot];
    if (count == 0) continue;
    std::vector<float> pk(count), pv(count), dpk(count), dpv(count), ks(count), vs(count);
    for (uint32_t j = 0; j < count; j++) {
      double kk = 0, vv = 0;
      for (uint32_t d = 0; d < h; d++) {
        const double s = states[uint64_t(start + j) * h + d];
        kk += double(pool[d]) * s;
        vv += double(pool[h + d]) * s;
      }
      ks[j] = f32(kk * scale);
      vs[j] = f32(vv * scale);
    }
    softmax_row(ks.data(), count);
    softmax_row(vs.data(), count);
    for (uint32_t j = 0; j < count; j++) {
      pk[j] = ks[j];
      pv[j] = vs[j];
      double dk = 0, dv = 0;
      for (uint32_t d = 0; d < h; d++) {
        const double s = states[uint64_t(start + j) * h + d];
        dk += double(d_keys[rec * h + d]) * s;
        dv += double(d_values[rec * h + d]) * s;
      }
      dpk[j] = f32(dk);
      dpv[j] = f32(dv);
    }
    double krs = 0, vrs = 0;
    for (uint32_t j = 0; j < count; j++) {
      krs += double(pk[j]) * double(dpk[j]);
      vrs += double(pv[j]) * double(dpv[j]);
    }
    for (uint32_t j = 0; j < count; j++) {
      const double dsk = double(pk[j]) * (double(dpk[j]) - krs);
      const double dsv = double(pv[j]) * (double(dpv[j]) - vrs);
      for (uint32_t d = 0; d < h; d++) {
        const double s = states[uint64_t(start + j) * h + d];
        const double ds = double(pk[j]) * double(d_keys[rec * h + d]) + double(pv[j]) * double(d_values[rec * h + d]) +
                          scale * (dsk * double(pool[d]) + dsv * double(pool[h + d]));
        float& dst = d_states[uint64_t(start + j) * h + d];
        dst = f32(double(dst) + ds);
        d_pool[d] = f32(double(d_pool[d]) + scale * dsk * s);
        d_pool[h + d] = f32(double(d_pool[h + d]) + scale * dsv * s);
      }
    }
  }
}

struct BackwardOut {
  std::vector<float> policy, value_prediction, d_sel_wq, d_sel_wk, d_pool, d_field_states, d_value_wv;
  double value_loss = 0;
};

// brainBackwardOracle (backward.ts:751-982) for a session's request.
// selection: [Q,R] mask; targets: [Q] or null; has_target/valence.
int backward(const ko_dims* d, const float* W, const uint32_t* token_rows, uint32_t token_rows_len, uint32_t slots,
             const uint32_t* token_ids, const uint32_t* field_roles, const uint32_t* schema_ids,
             const uint32_t* band_ids, const Active& a, const float* selection, const uint32_t* targets,
             int has_valence, double valence, BackwardOut& out) {
  const Layout L = layout_of(d);
  const uint32_t h = d->hidden, f = d->ffn, heads = d->heads, hd = d->head_dim;
  const uint64_t t = a.tokens.size();
  const uint32_t r = uint32_t(a.bank.size()), q = uint32_t(a.query.size());
  (void)slots;
  std::vector<uint32_t> rs(t), rc(t);
  for (uint32_t slot : a.records)
    for (uint32_t i = a.offset[slot]; i < a.offset[slot] + a.count[slot]; i++) { rs[i] = a.offset[slot]; rc[i] = a.count[slot]; }

  // forward with per-block saves (fieldEmbed as the forward)
  std::vector<float> x(t * h);
  const float* table = W + L.emb;
  for (uint64_t ti = 0; ti < t; ti++) {
    const uint32_t ft = a.tokens[ti];
    const uint32_t slot = ft >> 3, local = ft & 7;
    const uint32_t tid = token_ids[ft], rid = field_roles[ft];
    if (tid >= token_rows_len || rid >= token_rows_len) return -1;
    const uint32_t tok = token_rows[tid], role = token_rows[rid];
    const uint32_t schema = schema_ids[slot], band = band_ids[slot], stream = a.stream[slot];
    if (tok >= d->token_space || role >= d->field_space || schema >= d->schema_space || band >= d->band_space)
      return -1;
    for (uint32_t dd = 0; dd < h; dd++) {
      double value = 0;
      value += table[L.tb_token + uint64_t(tok) * h + dd];
      value += table[L.tb_field + uint64_t(role) * h + dd];
      value += table[L.tb_schema + uint64_t(schema) * h + dd];
      value += table[L.tb_band + uint64_t(band) * h + dd];
      value += table[L.tb_stream + uint64_t(stream) * h + dd];
      value += table[L.tb_pos + uint64_t(local) * h + dd];
      x[ti * h + dd] = f32(value);
    }
  }
  struct Saved { std::vector<float> q, k, v, p, h1; };
  const uint32_t kw_enc = 8;  // local windows are at most one record wide
  std::vector<Saved> enc(d->enc_blocks);
  std::vector<float> attn(t * h), ff(t * h);
  for (uint32_t b = 0; b < d->enc_blocks; b++) {
    const float* blk = W + L.enc + L.block * b;
    Saved& sv = enc[b];
    sv.q.resize(t * h); sv.k.resize(t * h); sv.v.resize(t * h); sv.p.assign(uint64_t(heads) * t * kw_enc, 0.f);
    sv.h1.resize(t * f);
    matmul(x.data(), blk, t, h, h, sv.q.data());
    matmul(x.data(), blk + h * h, t, h, h, sv.k.data());
    matmul(x.data(), blk + 2 * h * h, t, h, h, sv.v.data());
    attention_with_p(sv.q.data(), sv.k.data(), sv.v.data(), nullptr, t, t, h, heads, hd, rs.data(), rc.data(), kw_enc,
                     attn.data(), sv.p.data());
    add_inplace(x.data(), attn.data(), t * h);
    matmul(x.data(), blk + 3 * h * h, t, f, h, sv.h1.data());
    relu_inplace(sv.h1.data(), t * f);
    matmul(sv.h1.data(), blk + 3 * h * h + uint64_t(f) * h, t, h, f, ff.data());
    add_inplace(x.data(), ff.data(), t * h);
  }
  std::vector<float> bk(uint64_t(r) * h), bv(uint64_t(r) * h), qk(uint64_t(q) * h), qv(uint64_t(q) * h);
  const float* pool = W + L.pool;
  for (uint32_t i = 0; i < r; i++)
    pool_record(x.data(), a.offset[a.bank[i]], a.count[a.bank[i]], pool, h, bk.data() + uint64_t(i) * h,
                bv.data() + uint64_t(i) * h);
  for (uint32_t i = 0; i < q; i++)
    pool_record(x.data(), a.offset[a.query[i]], a.count[a.query[i]], pool, h, qk.data() + uint64_t(i) * h,
                qv.data() + uint64_t(i) * h);
  std::vector<Saved> mix(d->mixer_blocks);
  std::vector<float>& query = qv;
  std::vector<float> mattn(uint64_t(q) * h), mff(uint64_t(q) * h), zeros_qr(uint64_t(q) * r + 1, 0.f);
  for (uint32_t b = 0; b < d->mixer_blocks; b++) {
    const float* blk = W + L.mixer + L.block * b;
    Saved& sv = mix[b];
    sv.q.resize(uint64_t(q) * h); sv.k.resize(uint64_t(r) * h); sv.v.resize(uint64_t(r) * h);
    sv.p.assign(uint64_t(heads) * q * r + 1, 0.f); sv.h1.resize(uint64_t(q) * f);
    matmul(query.data(), blk, q, h, h, sv.q.data());
    matmul(bk.data(), blk + h * h, r, h, h, sv.k.data());
    matmul(bv.data(), blk + 2 * h * h, r, h, h, sv.v.data());
    attention_with_p(sv.q.data(), sv.k.data(), sv.v.data(), zeros_qr.data(), q, r, h, heads, hd, nullptr, nullptr, r,
                     mattn.data(), sv.p.data());
    add_inplace(query.data(), mattn.data(), uint64_t(q) * h);
    matmul(query.data(), blk + 3 * h * h, q, f, h, sv.h1.data());
    relu_inplace(sv.h1.data(), uint64_t(q) * f);
    matmul(sv.h1.data(), blk + 3 * h * h + uint64_t(f) * h, q, h, f, mff.data());
    add_inplace(query.data(), mff.data(), uint64_t(q) * h);
  }
  const std::vector<float>& qout = query;

  // the intent slot: selectorOracle under the selection mask
  std::vector<float> policy(uint64_t(q) * r + 1), gather(uint64_t(q) * h);
  std::vector<uint32_t> index(q + 1);
  selector(qout.data(), bk.data(), bv.data(), selection, W + L.sel_wq, W + L.sel_wk, q, r, h, nullptr, policy.data(),
           gather.data(), index.data());
  // offered: the mean bank value over what the grammar allows (backward.ts:834-843)
  std::vector<float> offered(uint64_t(q) * h, 0.f);
  std::vector<std::vector<uint32_t>> allowed(q);
  for (uint32_t i = 0; i < q; i++) {
    for (uint32_t j = 0; j < r; j++)
      if (double(selection[uint64_t(i) * r + j]) > -1e29) allowed[i].push_back(j);
    if (allowed[i].empty()) continue;
    for (uint32_t row : allowed[i])
      for (uint32_t dd = 0; dd < h; dd++)
        offered[uint64_t(i) * h + dd] = f32(double(offered[uint64_t(i) * h + dd]) + double(bv[uint64_t(row) * h + dd]));
    for (uint32_t dd = 0; dd < h; dd++)
      offered[uint64_t(i) * h + dd] = f32(double(offered[uint64_t(i) * h + dd]) / double(allowed[i].size()));
  }
  // value head: decisionHeadOracle with one class over [qout | gather | offered]
  const float* wv = W + L.value;
  const uint32_t hin = 3 * h;
  auto ctx = [&](uint32_t i, uint32_t dd) -> double {
    return dd < h ? qout[uint64_t(i) * h + dd]
                  : dd < 2 * h ? gather[uint64_t(i) * h + (dd - h)] : offered[uint64_t(i) * h + (dd - 2 * h)];
  };
  std::vector<float> pred(q + 1), dpred(q + 1, 0.f);
  for (uint32_t i = 0; i < q; i++) {
    double s = 0;
    for (uint32_t dd = 0; dd < hin; dd++) s += ctx(i, dd) * double(wv[dd]);
    pred[i] = f32(s);
  }
  double loss = 0;  // valueHeadLoss (backward.ts:49-62)
  if (has_valence && q) {
    for (uint32_t i = 0; i < q; i++) {
      const double e = double(pred[i]) - valence;
      loss += 0.5 * e * e;
      dpred[i] = f32(e / q);
    }
    loss /= q;
  }
  // decisionHeadBackward (backward.ts:459-506) for the value head, C = 1
  std::vector<float> dqo(uint64_t(q) * h), dig(uint64_t(q) * h), dag(uint64_t(q) * h), dwv(hin);
  for (uint32_t i = 0; i < q; i++)
    for (uint32_t dd = 0; dd < h; dd++) {
      const double dl = dpred[i];
      dqo[uint64_t(i) * h + dd] = f32(dl * double(wv[dd]));
      dig[uint64_t(i) * h + dd] = f32(dl * double(wv[h + dd]));
      dag[uint64_t(i) * h + dd] = f32(dl * double(wv[2 * h + dd]));
    }
  for (uint32_t dd = 0; dd < hin; dd++) {
    double s = 0;
    for (uint32_t i = 0; i < q; i++) s += double(dpred[i]) * ctx(i, dd);
    dwv[dd] = f32(s);
  }
  // dValue: the offered mean's gradient shared over its rows
  std::vector<float> dvalue(uint64_t(r) * h + 1, 0.f);
  for (uint32_t i = 0; i < q; i++) {
    if (allowed[i].empty()) continue;
    for (uint32_t row : allowed[i])
      for (uint32_t dd = 0; dd < h; dd++)
        dvalue[uint64_t(row) * h + dd] =
            f32(double(dvalue[uint64_t(row) * h + dd]) + double(dag[uint64_t(i) * h + dd]) / double(allowed[i].size()));
  }
  // selectorBackwardScores (backward.ts:293-336) for the intent slot
  std::vector<float> sq(uint64_t(q) * h), sk(uint64_t(r) * h);
  matmul(qout.data(), W + L.sel_wq, q, h, h, sq.data());
  matmul(bk.data(), W + L.sel_wk, r, h, h, sk.data());
  std::vector<float> dscore(uint64_t(q) * r + 1, 0.f), dpj(r + 1);
  for (uint32_t i = 0; i < q; i++) {
    const uint32_t raw = targets ? targets[i] : kInvalidU32;
    const bool valid = raw != kInvalidU32;
    const bool away = valid && raw >= 0x80000000u;
    const uint32_t target = away ? raw - 0x80000000u : raw;
    const double p_away = away && target < r ? double(policy[uint64_t(i) * r + target]) : 0.0;
    const double sc = away ? p_away / js_max(1 - p_away, 1e-6) : 0.0;
    double row_sum = 0;
    for (uint32_t j = 0; j < r; j++) {
      double s = 0;
      for (uint32_t dd = 0; dd < h; dd++) s += double(dig[uint64_t(i) * h + dd]) * double(bv[uint64_t(j) * h + dd]);
      dpj[j] = f32(s);
      row_sum += double(policy[uint64_t(i) * r + j]) * s;
    }
    for (uint32_t j = 0; j < r; j++) {
      const double pij = policy[uint64_t(i) * r + j];
      const double one = j == target ? 1.0 : 0.0;
      const double pg = !valid ? 0.0 : away ? sc * (one - pij) : pij - one;
      dscore[uint64_t(i) * r + j] = f32(pij * (double(dpj[j]) - row_sum) + pg);
    }
  }
  // selectorBackwardQkv (backward.ts:354-392), no gold filter for the intent slot
  const double hscale = 1 / std::sqrt(double(h));
  std::vector<float> dqp(uint64_t(q) * h), dkp(uint64_t(r) * h), dval2(uint64_t(r) * h);
  for (uint32_t i = 0; i < q; i++)
    for (uint32_t c = 0; c < h; c++) {
      double acc = 0;
      for (uint32_t j = 0; j < r; j++) acc += double(dscore[uint64_t(i) * r + j]) * double(sk[uint64_t(j) * h + c]);
      dqp[uint64_t(i) * h + c] = f32(acc * hscale);
    }
  for (uint32_t j = 0; j < r; j++)
    for (uint32_t c = 0; c < h; c++) {
      double ak = 0, av = 0;
      for (uint32_t i = 0; i < q; i++) {
        ak += double(dscore[uint64_t(i) * r + j]) * double(sq[uint64_t(i) * h + c]);
        av += double(policy[uint64_t(i) * r + j]) * double(dig[uint64_t(i) * h + c]);
      }
      dkp[uint64_t(j) * h + c] = f32(ak * hscale);
      dval2[uint64_t(j) * h + c] = f32(av);
    }
  // the accumulators start at zero (backward.ts:890-892): f32(0 + x) = x
  add_inplace(dvalue.data(), dval2.data(), uint64_t(r) * h);
  std::vector<float> dquery(uint64_t(q) * h), tmp_q(uint64_t(q) * h), dbk(uint64_t(r) * h);
  matmul_back_input(dqp.data(), W + L.sel_wq, q, h, h, tmp_q.data());
  dquery = dqo;
  add_inplace(dquery.data(), tmp_q.data(), uint64_t(q) * h);
  matmul_back_input(dkp.data(), W + L.sel_wk, r, h, h, dbk.data());
  std::vector<float> dbv = dvalue;
  out.d_sel_wq.assign(uint64_t(h) * h, 0.f);
  out.d_sel_wk.assign(uint64_t(h) * h, 0.f);
  matmul_back_weight(dqp.data(), qout.data(), q, h, h, out.d_sel_wq.data());
  matmul_back_weight(dkp.data(), bk.data(), r, h, h, out.d_sel_wk.data());

  // mixer blocks in reverse (backward.ts:925-941)
  std::vector<float> dh1r(uint64_t(q) * f), dffn(uint64_t(q) * h), dattn(uint64_t(q) * h), mdq(uint64_t(q) * h),
      mdk(uint64_t(r) * h), mdv(uint64_t(r) * h), t1(uint64_t(q) * h), t2(uint64_t(r) * h);
  for (int b = int(d->mixer_blocks) - 1; b >= 0; b--) {
    const float* blk = W + L.mixer + L.block * b;
    const Saved& sv = mix[b];
    matmul_back_input(dquery.data(), blk + 3 * h * h + uint64_t(f) * h, q, h, f, dh1r.data());
    for (uint64_t i = 0; i < uint64_t(q) * f; i++) dh1r[i] = sv.h1[i] > 0 ? dh1r[i] : 0.0f;
    matmul_back_input(dh1r.data(), blk + 3 * h * h, q, f, h, dffn.data());
    for (uint64_t i = 0; i < uint64_t(q) * h; i++) dattn[i] = f32(double(dquery[i]) + double(dffn[i]));
    attention_backward(dattn.data(), sv.q.data(), sv.k.data(), sv.v.data(), sv.p.data(), q, r, h, heads, hd, nullptr,
                       nullptr, r, mdq.data(), mdk.data(), mdv.data());
    dquery = dattn;
    matmul_back_input(mdq.data(), blk, q, h, h, t1.data());
    add_inplace(dquery.data(), t1.data(), uint64_t(q) * h);
    matmul_back_input(mdk.data(), blk + h * h, r, h, h, t2.data());
    add_inplace(dbk.data(), t2.data(), uint64_t(r) * h);
    matmul_back_input(mdv.data(), blk + 2 * h * h, r, h, h, t2.data());
    add_inplace(dbv.data(), t2.data(), uint64_t(r) * h);
  }
  // pool backward: bank records, then question records (zero key gradient)
  std::vector<float> dfs_bank(t * h, 0.f), dfs_query(t * h, 0.f), dpool_b(2 * h, 0.f), dpool_q(2 * h, 0.f);
  std::vector<float> zero_qk(uint64_t(q) * h + 1, 0.f);
  pool_backward(x.data(), a.bank, a, pool, dbk.data(), dbv.data(), h, dfs_bank.data(), dpool_b.data());
  pool_backward(x.data(), a.query, a, pool, zero_qk.data(), dquery.data(), h, dfs_query.data(), dpool_q.data());
  std::vector<float> dfs(t * h, 0.f), dpool(2 * h, 0.f);
  add_inplace(dfs.data(), dfs_bank.data(), t * h);
  add_inplace(dfs.data(), dfs_query.data(), t * h);
  add_inplace(dpool.data(), dpool_b.data(), 2 * h);
  add_inplace(dpool.data(), dpool_q.data(), 2 * h);
  // encoder blocks in reverse (backward.ts:956-968)
  std::vector<float> edh1(t * f), effn(t * h), eattn(t * h), edq(t * h), edk(t * h), edv(t * h), et(t * h);
  for (int b = int(d->enc_blocks) - 1; b >= 0; b--) {
    const float* blk = W + L.enc + L.block * b;
    const Saved& sv = enc[b];
    matmul_back_input(dfs.data(), blk + 3 * h * h + uint64_t(f) * h, t, h, f, edh1.data());
    for (uint64_t i = 0; i < t * f; i++) edh1[i] = sv.h1[i] > 0 ? edh1[i] : 0.0f;
    matmul_back_input(edh1.data(), blk + 3 * h * h, t, f, h, effn.data());
    for (uint64_t i = 0; i < t * h; i++) eattn[i] = f32(double(dfs[i]) + double(effn[i]));
    attention_backward(eattn.data(), sv.q.data(), sv.k.data(), sv.v.data(), sv.p.data(), t, t, h, heads, hd, rs.data(),
                       rc.data(), kw_enc, edq.data(), edk.data(), edv.data());
    dfs = eattn;
    matmul_back_input(edq.data(), blk, t, h, h, et.data());
    add_inplace(dfs.data(), et.data(), t * h);
    matmul_back_input(edk.data(), blk + h * h, t, h, h, et.data());
    add_inplace(dfs.data(), et.data(), t * h);
    matmul_back_input(edv.data(), blk + 2 * h * h, t, h, h, et.data());
    add_inplace(dfs.data(), et.data(), t * h);
  }
  out.policy.assign(policy.begin(), policy.begin() + uint64_t(q) * r);
  out.value_prediction.assign(pred.begin(), pred.begin() + q);
  out.value_loss = loss;
  out.d_pool = dpool;
  out.d_field_states = dfs;
  out.d_value_wv = dwv;
  return 0;
}

void mask_rule(uint32_t q, uint32_t r, const uint32_t* bank, const uint32_t* schema_ids, const uint32_t* band_ids,
               const uint32_t* schema_allow, const uint32_t* band_allow, float* mask) {
  for (uint32_t i = 0; i < q; i++) {
    uint32_t admitted = 0;
    for (uint32_t j = 0; j < r; j++) {
      const uint32_t slot = bank[j];
      const uint32_t s = schema_ids[slot], b = band_ids[slot];
      const bool ok = s < 256 && b < 32 && ((schema_allow[i * 8 + (s >> 5)] >> (s & 31)) & 1u) &&
                      ((band_allow[i] >> b) & 1u);
      if (ok) { admitted++; mask[uint64_t(i) * r + j] = 0.0f; }
      else mask[uint64_t(i) * r + j] = kNegInf;
    }
    if (!admitted)
      for (uint32_t j = 0; j < r; j++) mask[uint64_t(i) * r + j] = 0.0f;
  }
}

}  // namespace

extern "C" {

uint64_t ko_weight_count(const ko_dims* d) { return layout_of(d).total; }

uint64_t ko_weight_offset(const ko_dims* d, int which) {
  const Layout L = layout_of(d);
  switch (which) {
    case 0: return L.emb;
    case 1: return L.enc;
    case 2: return L.pool;
    case 3: return L.mixer;
    case 4: return L.sel_wq;
    case 5: return L.sel_wk;
    case 6: return L.decision;
    case 7: return L.value;
    default: return L.total;
  }
}

// createBrainForwardWeights (model.ts:233-265): one mulberry32 stream, in
// table order then block order.
void ko_create_weights(const ko_dims* d, uint32_t seed, float* out) {
  const Layout L = layout_of(d);
  Mulberry32 rand(seed);
  const uint64_t h = d->hidden, f = d->ffn;
  const uint32_t rows[6] = {d->token_space, d->field_space, d->schema_space, d->band_space, d->stream_space,
                            d->pos_space};
  uint64_t cursor = 0;
  for (int i = 0; i < 6; i++) {
    normal_table(uint64_t(rows[i]) * h, rand, 0.02, out + cursor);
    cursor += uint64_t(rows[i]) * h;
  }
  auto block = [&](float* dst) {
    xavier_uniform(h, h, rand, dst);
    xavier_uniform(h, h, rand, dst + h * h);
    xavier_uniform(h, h, rand, dst + 2 * h * h);
    xavier_uniform(f, h, rand, dst + 3 * h * h);
    xavier_uniform(h, f, rand, dst + 3 * h * h + f * h);
  };
  for (uint32_t b = 0; b < d->enc_blocks; b++) block(out + L.enc + L.block * b);
  normal_table(2 * h, rand, 0.02, out + L.pool);
  for (uint32_t b = 0; b < d->mixer_blocks; b++) block(out + L.mixer + L.block * b);
  xavier_uniform(h, h, rand, out + L.sel_wq);
  xavier_uniform(h, h, rand, out + L.sel_wk);
  xavier_uniform(d->route_kinds, 3 * h, rand, out + L.decision);
  xavier_uniform(1, 3 * h, rand, out + L.value);
}

void ko_mulberry32(uint32_t seed, uint32_t n, double* out) {
  Mulberry32 rand(seed);
  for (uint32_t i = 0; i < n; i++) out[i] = rand.next();
}

void ko_matmul(const float* x, const float* w, uint32_t rows, uint32_t out_dim, uint32_t in_dim, float* y) {
  matmul(x, w, rows, out_dim, in_dim, y);
}

void ko_softmax_row(float* v, uint32_t count) { softmax_row(v, count); }

int32_t ko_sample_row(const float* p, uint32_t count, double uniform) { return sample_row(p, count, uniform); }

uint32_t ko_compile_active(uint32_t slots, const uint32_t* token_ids, const uint32_t* band_ids,
                           const uint32_t* active_record_indices, uint32_t* active_tokens, uint32_t* rec_offset,
                           uint32_t* rec_count, uint32_t* stream_ids, uint32_t* bank_records,
                           uint32_t* query_records, uint32_t* r_out, uint32_t* q_out, uint32_t* active_count_out) {
  Active a;
  compile_active(slots, token_ids, band_ids, active_record_indices, a);
  std::memcpy(active_tokens, a.tokens.data(), a.tokens.size() * 4);
  std::memcpy(rec_offset, a.offset.data(), slots * 4ull);
  std::memcpy(rec_count, a.count.data(), slots * 4ull);
  std::memcpy(stream_ids, a.stream.data(), slots * 4ull);
  std::memcpy(bank_records, a.bank.data(), a.bank.size() * 4);
  std::memcpy(query_records, a.query.data(), a.query.size() * 4);
  *r_out = uint32_t(a.bank.size());
  *q_out = uint32_t(a.query.size());
  if (active_count_out) *active_count_out = uint32_t(a.records.size());
  return uint32_t(a.tokens.size());
}

int ko_forward(const ko_dims* d, const float* weights, const uint32_t* token_rows, uint32_t token_rows_len,
               uint32_t slots, const uint32_t* token_ids, const uint32_t* field_roles, const uint32_t* schema_ids,
               const uint32_t* band_ids, const uint32_t* active_record_indices, const float* mixer_mask,
               float* field_states, float* bank_keys, float* bank_values, float* query_keys,
               float* query_values_premix, float* query_output, const uint32_t* word_ids, float alpha) {
  Active a;
  compile_active(slots, token_ids, band_ids, active_record_indices, a);
  return forward(d, weights, token_rows, token_rows_len, slots, token_ids, field_roles, schema_ids, band_ids, a,
                 mixer_mask, field_states, bank_keys, bank_values, query_keys, query_values_premix, query_output,
                 word_ids, alpha);
}

void ko_selector(const float* query, const float* bank_keys, const float* bank_values, const float* mask,
                 const float* sel_wq, const float* sel_wk, uint32_t q, uint32_t r, uint32_t h,
                 const double* uniforms, float* p, float* gather, uint32_t* index) {
  selector(query, bank_keys, bank_values, mask, sel_wq, sel_wk, q, r, h, uniforms, p, gather, index);
}

void ko_selection_mask_rule(uint32_t q, uint32_t r, const uint32_t* bank_records, const uint32_t* schema_ids,
                            const uint32_t* band_ids, const uint32_t* schema_allow, const uint32_t* band_allow,
                            float* mask) {
  mask_rule(q, r, bank_records, schema_ids, band_ids, schema_allow, band_allow, mask);
}

void ko_batch_offsets(uint32_t frames, const uint64_t* rec_off, const uint32_t* token_ids, const uint32_t* band_ids,
                      uint64_t* p_off, uint64_t* q_off, uint64_t* r_off, uint64_t* t_off) {
  uint64_t pc = 0, qc = 0, rc = 0, tc = 0;
  for (uint32_t fi = 0; fi < frames; fi++) {
    p_off[fi] = pc; q_off[fi] = qc; if (r_off) r_off[fi] = rc; if (t_off) t_off[fi] = tc;
    uint64_t q = 0, n = rec_off[fi + 1] - rec_off[fi];
    for (uint64_t s = rec_off[fi]; s < rec_off[fi + 1]; s++) {
      q += band_ids[s] == kQueryBand;
      for (uint32_t l = 0; l < kRecordWidth; l++) tc += token_ids[s * kRecordWidth + l] != kPadToken;
    }
    const uint64_t r = n - q;
    qc += q; rc += r; pc += q * r;
  }
  p_off[frames] = pc; q_off[frames] = qc; if (r_off) r_off[frames] = rc; if (t_off) t_off[frames] = tc;
}

int ko_forward_batch(const ko_dims* d, const float* weights, const uint32_t* token_rows, uint32_t token_rows_len,
                     uint32_t frames, const uint64_t* rec_off, const uint32_t* token_ids, const uint32_t* field_roles,
                     const uint32_t* schema_ids, const uint32_t* band_ids, const uint32_t* schema_allow,
                     const uint32_t* band_allow, const double* uniforms, int threads, uint64_t* p_off,
                     uint64_t* q_off, float* p, uint32_t* index, float* query_output, const uint32_t* word_ids,
                     float alpha) {
  ko_batch_offsets(frames, rec_off, token_ids, band_ids, p_off, q_off, nullptr, nullptr);
  const Layout L = layout_of(d);
  const uint32_t h = d->hidden;
  std::atomic<int> failed{0};
  std::atomic<int64_t> next{0};
  auto worker = [&]() {
    for (int64_t fi = next++; fi < int64_t(frames); fi = next++) {
      const uint64_t r0 = rec_off[fi];
      const uint32_t slots = uint32_t(rec_off[fi + 1] - r0);
      const uint32_t* tid = token_ids + r0 * kRecordWidth;
      const uint32_t* rid = field_roles + r0 * kRecordWidth;
      const uint32_t* sid = schema_ids + r0;
      const uint32_t* bid = band_ids + r0;
      Active a;
      compile_active(slots, tid, bid, nullptr, a);
      const uint32_t r = uint32_t(a.bank.size()), q = uint32_t(a.query.size());
      const uint64_t qo = q_off[fi];
      if (q == 0) continue;
      if (r == 0) {  // consider() returns no selections for an empty bank (session.ts:133)
        for (uint32_t i = 0; i < q; i++) index[qo + i] = kInvalidU32;
        continue;
      }
      std::vector<float> bk(uint64_t(r) * h), bv(uint64_t(r) * h), qout(uint64_t(q) * h), mask(uint64_t(q) * r);
      if (forward(d, weights, token_rows, token_rows_len, slots, tid, rid, sid, bid, a, nullptr, nullptr, bk.data(),
                  bv.data(), nullptr, nullptr, qout.data(), word_ids ? word_ids + r0 * kRecordWidth : nullptr,
                  alpha) != 0) {
        failed = 1;
        continue;
      }
      if (query_output) std::memcpy(query_output + qo * h, qout.data(), qout.size() * sizeof(float));
      if (schema_allow) {
        // the rule is indexed by batch question; bank slots are frame-local
        mask_rule(q, r, a.bank.data(), sid, bid, schema_allow + qo * 8, band_allow + qo, mask.data());
      }
      selector(qout.data(), bk.data(), bv.data(), schema_allow ? mask.data() : nullptr, weights + L.sel_wq,
               weights + L.sel_wk, q, r, h, uniforms ? uniforms + qo : nullptr, p + p_off[fi], nullptr, index + qo);
    }
  };
  const int nt = threads > 0 ? threads : ko_max_threads();
  std::vector<std::thread> pool;
  for (int i = 1; i < nt; i++) pool.emplace_back(worker);
  worker();
  for (auto& th : pool) th.join();
  return failed ? -1 : 0;
}

int ko_backward(const ko_dims* d, const float* weights, const uint32_t* token_rows, uint32_t token_rows_len,
                uint32_t slots, const uint32_t* token_ids, const uint32_t* field_roles, const uint32_t* schema_ids,
                const uint32_t* band_ids, const uint32_t* active_record_indices, const float* selection,
                const uint32_t* targets, int has_valence, double valence, float* policy, float* value_prediction,
                double* value_loss, float* d_selector_wq, float* d_selector_wk, float* d_pool,
                float* d_field_states, float* d_value_wv) {
  Active a;
  compile_active(slots, token_ids, band_ids, active_record_indices, a);
  BackwardOut out;
  const int rc = backward(d, weights, token_rows, token_rows_len, slots, token_ids, field_roles, schema_ids, band_ids,
                          a, selection, targets, has_valence, valence, out);
  if (rc) return rc;
  std::memcpy(policy, out.policy.data(), out.policy.size() * 4);
  std::memcpy(value_prediction, out.value_prediction.data(), out.value_prediction.size() * 4);
  *value_loss = out.value_loss;
  std::memcpy(d_selector_wq, out.d_sel_wq.data(), out.d_sel_wq.size() * 4);
  std::memcpy(d_selector_wk, out.d_sel_wk.data(), out.d_sel_wk.size() * 4);
  std::memcpy(d_pool, out.d_pool.data(), out.d_pool.size() * 4);
  std::memcpy(d_field_states, out.d_field_states.data(), out.d_field_states.size() * 4);
  std::memcpy(d_value_wv, out.d_value_wv.data(), out.d_value_wv.size() * 4);
  return 0;
}

int ko_max_threads(void) {
  const unsigned n = std::thread::hardware_concurrency();
  return n ? int(n) : 1;
}

}  // extern "C"
