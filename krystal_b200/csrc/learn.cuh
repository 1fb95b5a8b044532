// learn.cuh — the update half of learnFromExperience (host/learn.ts:318-512)
// on the device, so a learn step needs no host round trip between the
// backward and the next forward.
//
//   k_learn_plan          the scalar plan over every frame of the (global)
//                         batch, every sum a running sum in frame order
//                         (:318-470): which frames count, the
//                         advantages, their mean and deviation, each frame's
//                         clipped step, the report's means;
//   k_learn_rows          the token and field rows' gradient sums when the
//                         tables are unfrozen (scatterEmbeddings, :242-263,
//                         in sum form) and which rows the batch touches;
//   k_learn_backup        the arrays the update may write, kept for the
//                         rollback (:401-425);
//   k_learn_update        critic, selector, pool and table rows (:427-470);
//   k_learn_health        parameterHealth (:187-205) before and after the update;
//   k_learn_settle        the rejection rule (:477-486) and the rollback.
//
// The reference subtracts each frame's step * gradient from its f32 arrays
// frame after frame; the update here subtracts the batch's f64 sums once
// (one rounding to f32 per element instead of one per frame), which moves
// nothing by more than the reference's 1e-4 gradient tolerance.
#pragma once
#include "common.cuh"

namespace kc {

struct LearnOpts {
  double lr, policy_scale, clip, max_abs, token_rate;
  int unfreeze_pool, unfreeze_tokens;
};

constexpr int kLearnRowWidth = 10;  // the 8 frame readings, the reward (NaN = none), answered (0 / 1)
// report: seen, actor moved, reinforced, discouraged, mean advantage, mean
// value loss, mean entropy, mean confidence, frames pending
constexpr int kLearnReport = 9;
// result: applied, rejected (0 none, 1 non-finite, 2 parameter limit),
// finite, then the health maxima: table rows, selector, value head, pool,
// selector Wq, selector Wk; then the rows touched
constexpr int kLearnResult = 10;
constexpr int kHealthGroups = 5;  // rows, wq, wk, value, pool

// plan_update's arithmetic in the reference's order. The rows stream
// through shared memory in chunks of kPlanChunk frames; the per-frame
// outputs (value weight, pending, step) are written by all threads, and the
// running sums, whose order matters, by thread 0 alone from shared memory.
constexpr int kPlanChunk = 1024;
constexpr int kPlanThreads = 256;
constexpr size_t kPlanSmem = size_t(kPlanChunk) * kLearnRowWidth * 8;

__device__ __forceinline__ bool plan_used(const double* r) {  // a reward, and something to choose (:319-324)
  return !isnan(r[8]) && r[0] != 0.0 && r[1] != 0.0;
}
__device__ __forceinline__ bool plan_pending(const double* r) {  // answered, with a finite advantage (:374)
  return plan_used(r) && r[9] > 0.0 && isfinite(r[8] - r[2]);
}

__global__ void __launch_bounds__(kPlanThreads) k_learn_plan(const double* __restrict__ rows, uint32_t frames,
                                                             LearnOpts o, double* __restrict__ step,
                                                             double* __restrict__ value_weight,
                                                             double* __restrict__ pending,
                                                             double* __restrict__ report) {
  extern __shared__ double pr[];  // [kPlanChunk][kLearnRowWidth]
  __shared__ double s_mean, s_dev;
  __shared__ uint32_t s_n, s_moved, s_reinforced, s_discouraged;
  const int tid = threadIdx.x;
  double adv_total = 0.0, loss_total = 0.0, ent_total = 0.0, ent_rows = 0.0, conf_total = 0.0, conf_rows = 0.0;
  double pend_total = 0.0, var_total = 0.0;
  uint32_t seen = 0, n = 0;
  if (tid == 0) s_reinforced = s_discouraged = 0;
  auto stage = [&](uint32_t c0, uint32_t nc) {
    __syncthreads();
    for (uint32_t i = tid; i < nc * kLearnRowWidth; i += kPlanThreads) pr[i] = rows[uint64_t(c0) * kLearnRowWidth + i];
    __syncthreads();
  };
  // pass 1: which frames count, the report's running sums, the advantages' sum
  for (uint32_t c0 = 0; c0 < frames; c0 += kPlanChunk) {
    const uint32_t nc = min(uint32_t(kPlanChunk), frames - c0);
    stage(c0, nc);
    for (uint32_t i = tid; i < nc; i += kPlanThreads) {
      const double* r = pr + i * kLearnRowWidth;
      step[c0 + i] = 0.0;
      value_weight[c0 + i] = plan_used(r) ? 1.0 : 0.0;
      pending[c0 + i] = plan_pending(r) ? 1.0 : 0.0;
    }
    if (tid == 0)
      for (uint32_t i = 0; i < nc; i++) {
        const double* r = pr + i * kLearnRowWidth;
        if (!plan_used(r)) continue;
        const double adv = r[8] - r[2];
        seen++;
        adv_total += adv;
        loss_total += r[3];
        ent_total += r[4];
        ent_rows += r[5];
        conf_total += r[6];
        conf_rows += r[7];
        if (plan_pending(r)) {
          pend_total += adv;
          n++;
        }
      }
  }
  if (tid == 0) {
    s_n = n;
    s_mean = n ? pend_total / double(n) : 0.0;
  }
  __syncthreads();
  const uint32_t n_all = s_n;
  const double mean = s_mean;
  // pass 2: the deviation, (a - mean)^2 summed in frame order
  if (n_all) {
    for (uint32_t c0 = 0; c0 < frames; c0 += kPlanChunk) {
      const uint32_t nc = min(uint32_t(kPlanChunk), frames - c0);
      stage(c0, nc);
      if (tid == 0)
        for (uint32_t i = 0; i < nc; i++) {
          const double* r = pr + i * kLearnRowWidth;
          if (!plan_pending(r)) continue;
          const double d = (r[8] - r[2]) - mean;
          var_total += d * d;
        }
    }
    if (tid == 0) {
      s_dev = sqrt(var_total / double(n_all));
      s_moved = s_dev > 1e-6 ? 1u : 0u;  // a batch where everything went equally well pushes nothing (:447-451)
    }
  } else if (tid == 0) {
    s_dev = 0.0;
    s_moved = 0u;
  }
  __syncthreads();
  const bool moved = s_moved != 0u;
  const double deviation = s_dev;
  // pass 3: each pending frame's clipped step
  if (moved)
    for (uint32_t c0 = 0; c0 < frames; c0 += kPlanChunk) {
      const uint32_t nc = min(uint32_t(kPlanChunk), frames - c0);
      stage(c0, nc);
      uint32_t up = 0, down = 0;
      for (uint32_t i = tid; i < nc; i += kPlanThreads) {
        const double* r = pr + i * kLearnRowWidth;
        if (!plan_pending(r)) continue;
        const double st = fmin(o.clip, fmax(-o.clip, ((r[8] - r[2]) - mean) / deviation));
        step[c0 + i] = (o.lr * o.policy_scale * st) / double(n_all);
        up += st > 0.0;
        down += st < 0.0;
      }
      if (up) atomicAdd(&s_reinforced, up);
      if (down) atomicAdd(&s_discouraged, down);
    }
  __syncthreads();
  if (tid == 0) {
    report[0] = seen;
    report[1] = moved ? 1.0 : 0.0;
    report[2] = s_reinforced;
    report[3] = s_discouraged;
    report[4] = seen ? adv_total / double(seen) : 0.0;
    report[5] = seen ? loss_total / double(seen) : 0.0;
    report[6] = ent_rows != 0.0 ? ent_total / ent_rows : 0.0;
    report[7] = conf_rows != 0.0 ? conf_total / conf_rows : 0.0;
    report[8] = n_all;
  }
}

// One warp per 32 consecutive tokens of the last batch differentiated, lane l
// owning columns 4l..4l+3: row_sums[token row] and row_sums[token_space +
// field row] gain step[frame] * dFieldStates[t] for tokens of pending frames,
// and both rows are marked touched. A field row shared by consecutive tokens
// (the session's default role is row 0) is summed in registers and added
// once per run. The f64 atomics make the order of a row's additions, and so
// its last bits, vary from run to run.
__global__ void __launch_bounds__(256) k_learn_rows(const uint64_t* __restrict__ t_off, uint32_t frames,
                                                    const uint32_t* __restrict__ tok_recpos,
                                                    const uint32_t* __restrict__ token_ids,
                                                    const uint32_t* __restrict__ field_roles,
                                                    const uint32_t* __restrict__ token_rows,
                                                    const double* __restrict__ step,
                                                    const double* __restrict__ pending,
                                                    const float* __restrict__ dfs, uint64_t T, uint32_t token_space,
                                                    double* __restrict__ row_sums, double* __restrict__ touched) {
  const uint64_t t0 = (uint64_t(blockIdx.x) * 8 + (threadIdx.x >> 5)) * 32;
  if (t0 >= T) return;
  const int lane = threadIdx.x & 31, d = lane * 4;
  const uint64_t t1 = t0 + 32 < T ? t0 + 32 : T;
  // the frame of t0: the last f with t_off[f] <= t0
  uint32_t lo = 0, hi = frames;
  while (hi - lo > 1) {
    const uint32_t mid = (lo + hi) / 2;
    if (t_off[mid] <= t0) lo = mid; else hi = mid;
  }
  uint32_t f = lo;
  uint32_t run_row = KC_INVALID;
  double acc[4] = {0.0, 0.0, 0.0, 0.0};
  auto flush = [&]() {
    if (run_row == KC_INVALID) return;
    double* dst = row_sums + uint64_t(run_row) * KC_H + d;
#pragma unroll
    for (int e = 0; e < 4; e++) {
      atomicAdd(dst + e, acc[e]);
      acc[e] = 0.0;
    }
    if (lane == 0) touched[run_row] = 1.0;
    run_row = KC_INVALID;
  };
  for (uint64_t t = t0; t < t1; t++) {
    while (f + 1 < frames && t_off[f + 1] <= t) f++;
    if (pending[f] == 0.0) continue;
    const uint32_t rp = tok_recpos[t];
    const uint64_t slot = uint64_t(rp >> 3) * KC_RW + (rp & 7u);
    const uint32_t tr = token_rows[token_ids[slot]];
    const uint32_t fr = token_space + token_rows[field_roles[slot]];
    const double s = step[f];
    const float4 g = *reinterpret_cast<const float4*>(dfs + t * KC_H + d);
    const double v[4] = {s * double(g.x), s * double(g.y), s * double(g.z), s * double(g.w)};
    double* tdst = row_sums + uint64_t(tr) * KC_H + d;
#pragma unroll
    for (int e = 0; e < 4; e++) atomicAdd(tdst + e, v[e]);
    if (lane == 0) touched[tr] = 1.0;
    if (fr != run_row) {
      flush();
      run_row = fr;
    }
#pragma unroll
    for (int e = 0; e < 4; e++) acc[e] += v[e];
  }
  flush();
}

struct LearnApplyArgs {
  float* page;
  uint64_t off_swq, off_swk, off_val, off_pool, tb_token;  // page offsets (floats)
  uint32_t rows;             // token_space + field_space: the rows the tables hold
  const double* sums;        // [wq H*H | wk H*H | pool 2H | value 3H]
  const double* row_sums;    // [rows, H] or null
  const double* touched;     // [rows] (> 0 touched) or null
  const double* report;      // k_learn_plan's
  LearnOpts o;
  float* backup;             // [wq | wk | value | pool | rows x H]
  // per group max |x| as float bits, then non-finite flags: before the
  // update [0, 2G), after it [2G, 4G)
  unsigned* health;
  double* result;            // [kLearnResult]
};

// Elements of the groups the update may write, in backup order.
__device__ __forceinline__ uint64_t learn_elems(const LearnApplyArgs& a) {
  return 2ull * KC_H * KC_H + 3 * KC_H + 2 * KC_H + (a.row_sums ? uint64_t(a.rows) * KC_H : 0);
}

// Element e of the backup order -> its page offset, or ~0 for a table row
// the batch does not touch.
__device__ __forceinline__ uint64_t learn_page_off(const LearnApplyArgs& a, uint64_t e, int* group) {
  const uint64_t hh = uint64_t(KC_H) * KC_H;
  if (e < hh) { *group = 1; return a.off_swq + e; }
  e -= hh;
  if (e < hh) { *group = 2; return a.off_swk + e; }
  e -= hh;
  if (e < 3 * KC_H) { *group = 3; return a.off_val + e; }
  e -= 3 * KC_H;
  if (e < 2 * KC_H) { *group = 4; return a.off_pool + e; }
  e -= 2 * KC_H;
  *group = 0;
  return a.touched[e / KC_H] > 0.0 ? a.tb_token + e : ~0ull;
}

__global__ void k_learn_backup(LearnApplyArgs a) {
  const uint64_t n = learn_elems(a);
  for (uint64_t e = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < n; e += uint64_t(gridDim.x) * blockDim.x) {
    int g;
    const uint64_t o = learn_page_off(a, e, &g);
    if (o != ~0ull) a.backup[e] = a.page[o];
  }
}

// f32(w - delta) in f64, as the reference's Float32Array writes round.
__global__ void k_learn_update(LearnApplyArgs a) {
  const double seen = a.report[0];
  const bool moved = a.report[1] != 0.0;
  const uint64_t n = learn_elems(a), hh = uint64_t(KC_H) * KC_H;
  for (uint64_t e = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < n; e += uint64_t(gridDim.x) * blockDim.x) {
    int g;
    const uint64_t o = learn_page_off(a, e, &g);
    if (o == ~0ull) continue;
    double delta;
    bool write = false;
    if (g == 1 || g == 2) {  // selector: sum_f step_f dW_f
      write = moved;
      delta = a.sums[e];
    } else if (g == 3) {     // critic: lr * sum dWv / seen
      write = seen != 0.0;
      delta = (a.o.lr * a.sums[2 * hh + 2 * KC_H + (e - 2 * hh)]) / seen;
    } else if (g == 4) {     // pool, when unfrozen
      write = moved && a.o.unfreeze_pool;
      delta = a.sums[2 * hh + (e - 2 * hh - 3 * KC_H)];
    } else {                 // a touched table row, when unfrozen
      write = moved && a.o.unfreeze_tokens;
      delta = a.o.token_rate * a.row_sums[e - 2 * hh - 5 * KC_H];
    }
    if (write) a.page[o] = __double2float_rn(double(a.page[o]) - delta);
  }
}

// max |x| per group (rows, wq, wk, value, pool) and whether any is not
// finite, into health[0, 2G) (which = 0, before the update) or [2G, 4G).
__global__ void __launch_bounds__(256) k_learn_health(LearnApplyArgs a, int which) {
  __shared__ unsigned mx[kHealthGroups], bad[kHealthGroups];
  if (threadIdx.x < kHealthGroups) mx[threadIdx.x] = bad[threadIdx.x] = 0u;
  __syncthreads();
  float m[kHealthGroups] = {0.f, 0.f, 0.f, 0.f, 0.f};
  unsigned nf[kHealthGroups] = {0u, 0u, 0u, 0u, 0u};
  const uint64_t n = learn_elems(a);
  for (uint64_t e = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < n; e += uint64_t(gridDim.x) * blockDim.x) {
    int g;
    const uint64_t o = learn_page_off(a, e, &g);
    if (o == ~0ull) continue;
    const float v = fabsf(a.page[o]);
    if (!(v <= 3.402823466e38f)) nf[g] = 1u;  // NaN or infinite
    else m[g] = fmaxf(m[g], v);
  }
#pragma unroll
  for (int g = 0; g < kHealthGroups; g++) {
    if (m[g] > 0.f) atomicMax(&mx[g], __float_as_uint(m[g]));
    if (nf[g]) bad[g] = 1u;
  }
  __syncthreads();
  unsigned* h = a.health + which * 2 * kHealthGroups;
  if (threadIdx.x < kHealthGroups) {
    atomicMax(&h[threadIdx.x], mx[threadIdx.x]);
    if (bad[threadIdx.x]) atomicOr(&h[kHealthGroups + threadIdx.x], 1u);
  }
}

// Health words -> maxima (a non-finite group reads as infinity, as the
// host's max-abs does) and whether every group is finite.
__device__ __forceinline__ bool learn_health_values(const unsigned* h, double* hv) {
  bool finite = true;
#pragma unroll
  for (int g = 0; g < kHealthGroups; g++) {
    const bool nf = h[kHealthGroups + g] != 0u;
    finite = finite && !nf;
    hv[g] = nf ? INFINITY : double(__uint_as_float(h[g]));
  }
  return finite;
}

// The rejection rule and, on a rejection, the rollback; the result, whose
// health is that of the arrays as they are left (:496-511). Every thread
// reads the same health words, so all take the same decision.
__global__ void k_learn_settle(LearnApplyArgs a) {
  double hv[kHealthGroups], hb[kHealthGroups];
  const bool finite = learn_health_values(a.health + 2 * kHealthGroups, hv);
  const bool finite_before = learn_health_values(a.health, hb);
  const double sel = fmax(hv[1], hv[2]);
  const bool over = hv[0] > a.o.max_abs || sel > a.o.max_abs || hv[3] > a.o.max_abs || hv[4] > a.o.max_abs;
  const int rejected = !finite ? 1 : over ? 2 : 0;
  const uint64_t n = learn_elems(a);
  if (rejected)
    for (uint64_t e = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < n;
         e += uint64_t(gridDim.x) * blockDim.x) {
      int g;
      const uint64_t o = learn_page_off(a, e, &g);
      if (o != ~0ull) a.page[o] = a.backup[e];
    }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    const double* hf = rejected ? hb : hv;
    a.result[0] = (a.report[0] > 0.0 && !rejected) ? 1.0 : 0.0;
    a.result[1] = rejected;
    a.result[2] = (rejected ? finite_before : finite) ? 1.0 : 0.0;
    a.result[3] = hf[0];
    a.result[4] = fmax(hf[1], hf[2]);
    a.result[5] = hf[3];
    a.result[6] = hf[4];
    a.result[7] = hf[1];
    a.result[8] = hf[2];
    double rows = 0.0;
    if (a.touched)
      for (uint32_t r = 0; r < a.rows; r++) rows += a.touched[r] > 0.0 ? 1.0 : 0.0;
    a.result[9] = rows;
  }
}

}  // namespace kc
