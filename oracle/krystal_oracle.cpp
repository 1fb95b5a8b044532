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
void attention(const float* q, const float* k, const float* v, const float* mask, uint64_t q_rows, uint64_t k_rows,
               uint32_t h, uint32_t heads, uint32_t head_dim, const uint32_t* local_start,
               const uint32_t* local_count, float* out) {
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
            float* query_output) {
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
              attn.data());
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
               float* query_values_premix, float* query_output) {
  Active a;
  compile_active(slots, token_ids, band_ids, active_record_indices, a);
  return forward(d, weights, token_rows, token_rows_len, slots, token_ids, field_roles, schema_ids, band_ids, a,
                 mixer_mask, field_states, bank_keys, bank_values, query_keys, query_values_premix, query_output);
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
                     uint64_t* q_off, float* p, uint32_t* index, float* query_output) {
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
                  bv.data(), nullptr, nullptr, qout.data()) != 0) {
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

int ko_max_threads(void) {
  const unsigned n = std::thread::hardware_concurrency();
  return n ? int(n) : 1;
}

}  // extern "C"
