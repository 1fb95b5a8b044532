// pack.cuh — ragged frame packing on the GPU.
//
// The reference compiles every frame on the host, one at a time
// (compileActiveFrame, packages/krystal/src/forward/masks.ts:65-101, called
// from packHostFrame, host/frame.ts:114). Here a whole batch of frames is
// compiled at once from the flat per-record arrays plus the record-offset
// table, with three kernels:
//
//   k_frame_scan     one CTA per frame: counts each record's non-PAD tokens,
//                    classifies question / bank (band 5, masks.ts:86), and
//                    block-scans both within the frame; validates ids.
//   k_frame_offsets  one CTA: scans the per-frame totals into the batch's
//                    token / question / bank / p offset tables.
//   k_record_rows    one CTA per frame: writes the compact token list
//                    (record-major, masks.ts:73-85), each record's compact
//                    range (recordRanges, masks.ts:120-133) and the bank and
//                    question row lists (masks.ts:89-90) at batch offsets.
#pragma once
#include "common.cuh"

namespace kc {

// Per-record scratch written by k_frame_scan.
//   x: compact token offset of the record inside its frame
//   y: (row_local << 5) | (is_query << 4) | token_count
struct FrameTotals {
  unsigned long long t, q, r, p;  // batch totals
  unsigned int max_r, max_q, bad, bad_where;
};

// error codes written to FrameTotals::bad
enum : uint32_t {
  kBadNone = 0,
  kBadTokenId = 1,    // a token id with no entry in token_rows
  kBadTokenRow = 2,   // a projected token row outside the token table
  kBadRoleId = 3,
  kBadRoleRow = 4,
  kBadSchema = 5,
  kBadBand = 6,
  kBadEmptyFrame = 7, // a frame without records
  kBadBank = 8,       // a frame's bank beyond the supported maximum
};

__device__ __forceinline__ void flag_bad(FrameTotals* tot, uint32_t code, uint32_t where) {
  if (atomicCAS(&tot->bad, 0u, code) == 0u) tot->bad_where = where;
}

template <int NT>
__global__ void __launch_bounds__(NT) k_frame_scan(
    const uint64_t* __restrict__ rec_off, uint32_t frames, const uint32_t* __restrict__ token_ids,
    const uint32_t* __restrict__ field_roles, const uint32_t* __restrict__ schema_ids,
    const uint32_t* __restrict__ band_ids, const uint32_t* __restrict__ token_rows, uint32_t token_rows_len,
    uint32_t token_space, uint32_t field_space, uint32_t schema_space, uint32_t band_space, uint32_t max_bank,
    uint2* __restrict__ rec_meta, uint32_t* __restrict__ frame_t, uint32_t* __restrict__ frame_q,
    uint32_t* __restrict__ frame_r, FrameTotals* tot) {
  __shared__ uint32_t tmp[NT / 32];
  const uint32_t f = blockIdx.x;
  if (f >= frames) return;
  const uint64_t r0 = rec_off[f], r1 = rec_off[f + 1];
  const uint32_t n = uint32_t(r1 - r0);
  if (n == 0 && threadIdx.x == 0) flag_bad(tot, kBadEmptyFrame, f);
  uint32_t tok_base = 0, q_base = 0;
  for (uint32_t c = 0; c < n; c += NT) {
    const uint32_t s = c + threadIdx.x;
    uint32_t cnt = 0, isq = 0;
    if (s < n) {
      const uint64_t g = r0 + s;
      const uint4* tp = reinterpret_cast<const uint4*>(token_ids + g * KC_RW);
      const uint4 a = tp[0], b = tp[1];
      const uint32_t ids[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
      for (int l = 0; l < 8; l++) {
        if (ids[l] == 0u) continue;  // PAD
        cnt++;
        if (ids[l] >= token_rows_len) { flag_bad(tot, kBadTokenId, uint32_t(g)); continue; }
        if (token_rows[ids[l]] >= token_space) flag_bad(tot, kBadTokenRow, uint32_t(g));
        const uint32_t role = field_roles[g * KC_RW + l];
        if (role >= token_rows_len) { flag_bad(tot, kBadRoleId, uint32_t(g)); continue; }
        if (token_rows[role] >= field_space) flag_bad(tot, kBadRoleRow, uint32_t(g));
      }
      const uint32_t band = band_ids[g];
      if (schema_ids[g] >= schema_space) flag_bad(tot, kBadSchema, uint32_t(g));
      if (band >= band_space) flag_bad(tot, kBadBand, uint32_t(g));
      isq = band == KC_QUERY_BAND_ID;
    }
    uint32_t total;
    const uint32_t ex = block_excl_scan<NT, uint32_t>((cnt << 16) | isq, &total, tmp);
    if (s < n) {
      const uint32_t tok_local = tok_base + (ex >> 16);
      const uint32_t q_local = q_base + (ex & 0xffffu);
      const uint32_t row_local = isq ? q_local : (s - q_local);
      rec_meta[r0 + s] = make_uint2(tok_local, (row_local << 5) | (isq << 4) | cnt);
    }
    tok_base += total >> 16;
    q_base += total & 0xffffu;
  }
  if (threadIdx.x == 0) {
    frame_t[f] = tok_base;
    frame_q[f] = q_base;
    frame_r[f] = n - q_base;
    if (n - q_base > max_bank) flag_bad(tot, kBadBank, f);
  }
}

// One CTA of NT threads scans all frames. Offsets are [frames+1] each.
template <int NT>
__global__ void __launch_bounds__(NT) k_frame_offsets(
    uint32_t frames, const uint32_t* __restrict__ frame_t, const uint32_t* __restrict__ frame_q,
    const uint32_t* __restrict__ frame_r, uint64_t* __restrict__ t_off, uint64_t* __restrict__ q_off,
    uint64_t* __restrict__ r_off, uint64_t* __restrict__ p_off, FrameTotals* tot) {
  __shared__ unsigned long long tmp[NT / 32];
  unsigned long long bt = 0, bq = 0, br = 0, bp = 0;
  uint32_t mr = 0, mq = 0;
  for (uint32_t c = 0; c < frames; c += NT) {
    const uint32_t f = c + threadIdx.x;
    unsigned long long t = 0, q = 0, r = 0;
    if (f < frames) { t = frame_t[f]; q = frame_q[f]; r = frame_r[f]; mr = max(mr, uint32_t(r)); mq = max(mq, uint32_t(q)); }
    unsigned long long tt, tq, tr, tp;
    const unsigned long long et = block_excl_scan<NT, unsigned long long>(t, &tt, tmp);
    const unsigned long long eq = block_excl_scan<NT, unsigned long long>(q, &tq, tmp);
    const unsigned long long er = block_excl_scan<NT, unsigned long long>(r, &tr, tmp);
    const unsigned long long ep = block_excl_scan<NT, unsigned long long>(q * r, &tp, tmp);
    if (f < frames) { t_off[f] = bt + et; q_off[f] = bq + eq; r_off[f] = br + er; p_off[f] = bp + ep; }
    bt += tt; bq += tq; br += tr; bp += tp;
  }
  // max over threads
  for (int o = 16; o; o >>= 1) {
    mr = max(mr, __shfl_xor_sync(0xffffffffu, mr, o));
    mq = max(mq, __shfl_xor_sync(0xffffffffu, mq, o));
  }
  if ((threadIdx.x & 31) == 0) { atomicMax(&tot->max_r, mr); atomicMax(&tot->max_q, mq); }
  if (threadIdx.x == 0) {
    t_off[frames] = bt; q_off[frames] = bq; r_off[frames] = br; p_off[frames] = bp;
    tot->t = bt; tot->q = bq; tot->r = br; tot->p = bp;
  }
}

// Per compact token: (global record << 3) | position in the record.
// Per record: global compact start (the record's range is start..start+count).
// Per bank row: global record; per question row: global record and frame.
template <int NT>
__global__ void __launch_bounds__(NT) k_record_rows(
    const uint64_t* __restrict__ rec_off, uint32_t frames, const uint32_t* __restrict__ token_ids,
    const uint2* __restrict__ rec_meta, const uint64_t* __restrict__ t_off, const uint64_t* __restrict__ q_off,
    const uint64_t* __restrict__ r_off, uint32_t* __restrict__ tok_recpos, uint32_t* __restrict__ rec_start,
    uint32_t* __restrict__ rec_row, uint32_t* __restrict__ bank_rec, uint32_t* __restrict__ query_rec,
    uint32_t* __restrict__ query_frame, uint32_t* __restrict__ bank_frame) {
  const uint32_t f = blockIdx.x;
  if (f >= frames) return;
  const uint64_t r0 = rec_off[f], r1 = rec_off[f + 1];
  const uint32_t tb = uint32_t(t_off[f]), qb = uint32_t(q_off[f]), rb = uint32_t(r_off[f]);
  for (uint64_t g = r0 + threadIdx.x; g < r1; g += NT) {
    const uint2 m = rec_meta[g];
    const uint32_t start = tb + m.x;
    const uint32_t isq = (m.y >> 4) & 1u, row_local = m.y >> 5;
    rec_start[g] = start;
    const uint4* tp = reinterpret_cast<const uint4*>(token_ids + g * KC_RW);
    const uint4 a = tp[0], b = tp[1];
    const uint32_t ids[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    uint32_t k = 0;
#pragma unroll
    for (uint32_t l = 0; l < 8; l++)
      if (ids[l] != 0u) tok_recpos[start + k++] = (uint32_t(g) << 3) | l;
    if (isq) {
      const uint32_t row = qb + row_local;
      rec_row[g] = row | 0x80000000u;
      query_rec[row] = uint32_t(g);
      query_frame[row] = f;
    } else {
      const uint32_t row = rb + row_local;
      rec_row[g] = row;
      bank_rec[row] = uint32_t(g);
      bank_frame[row] = f;
    }
  }
}

}  // namespace kc
