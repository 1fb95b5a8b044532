// stream.cuh — the streaming packer: frames arrive one at a time, leave in
// rolling batches (included by krystal_cuda.cu; host code only).
//
// A session thinks about one frame per turn (host/session.ts:128-181); an
// interactive host with many creatures sees those turns arrive continuously.
// kc_stream turns that arrival stream into packed ragged batches:
//
//   push   copies one frame's active records (compileActiveFrame's walk,
//          masks.ts:73-74) into the open pinned staging buffer and validates
//          it there, so a malformed frame is refused alone instead of
//          failing the batch it would have joined;
//   flush  seals the open buffer and queues it; a worker thread runs sealed
//          buffers back to back through the batch path (H2D from pinned
//          memory, GPU packing, encode, select, D2H into the buffer's pinned
//          result arrays), while the caller keeps pushing into the next
//          buffer;
//   poll   hands back the oldest finished batch: its ticket range, per-frame
//          offsets, p and indices, and the steady-clock times at which it was
//          sealed and finished.
//
// Buffers cycle free -> open -> sealed -> running -> done -> handed out; the
// batch handed out by a poll stays readable until the next poll.

#include <chrono>
#include <condition_variable>
#include <deque>
#include <thread>

namespace {

double steady_ms() {
  return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

enum BufState { kFree = 0, kOpen, kSealed, kRunning, kDone, kHanded };

struct StreamBuf {
  // staging (pinned host)
  uint64_t* rec_off = nullptr;   // [max_frames + 1]
  uint32_t *tok = nullptr, *role = nullptr, *sch = nullptr, *band = nullptr;  // [max_records(*8)]
  uint32_t *sa = nullptr, *ba = nullptr;  // rule per question: [max_records * 8], [max_records]
  // results (pinned host)
  float* p = nullptr;
  uint32_t* index = nullptr;
  uint64_t *p_off = nullptr, *q_off = nullptr;
  // contents
  uint32_t frames = 0;
  uint64_t records = 0, questions = 0, p_total = 0;
  bool has_rule = false;
  uint64_t first_ticket = 0;
  BufState state = kFree;
  kc_status status = KC_OK;
  std::string err;
  double seal_ms = 0, done_ms = 0;
};

}  // namespace

struct kc_stream {
  kc_handle* h = nullptr;
  uint32_t max_frames = 0;
  uint64_t max_records = 0, max_p = 0;
  std::vector<StreamBuf> bufs;
  int open = -1;
  std::deque<int> queue;   // sealed and running, in order
  std::deque<int> done;    // finished, in order
  int handed = -1;
  uint64_t next_ticket = 0;
  std::mutex mu;
  std::condition_variable cv;
  std::thread worker;
  bool stop = false;
  std::string err;
};

namespace {

kc_status stream_fail(kc_stream* s, kc_status st, const std::string& msg) {
  s->err = msg;
  return st;
}

void free_buf(StreamBuf& b) {
  void* ptrs[] = {b.rec_off, b.tok, b.role, b.sch, b.band, b.sa, b.ba, b.p, b.index, b.p_off, b.q_off};
  for (void* p : ptrs)
    if (p) cudaFreeHost(p);
}

// The worker: runs sealed buffers in order through the batch path.
void stream_worker(kc_stream* s) {
  cudaSetDevice(s->h->device);
  for (;;) {
    int idx;
    {
      std::unique_lock<std::mutex> lk(s->mu);
      s->cv.wait(lk, [&] {
        if (s->stop) return true;
        for (int i : s->queue)
          if (s->bufs[i].state == kSealed) return true;
        return false;
      });
      if (s->stop) return;
      idx = -1;
      for (int i : s->queue)
        if (s->bufs[i].state == kSealed) { idx = i; break; }
      s->bufs[idx].state = kRunning;
    }
    StreamBuf& b = s->bufs[idx];
    kc_batch_view bv{};
    bv.frames = b.frames;
    bv.records = b.records;
    bv.rec_off = b.rec_off;
    bv.token_ids = b.tok;
    bv.field_roles = b.role;
    bv.schema_ids = b.sch;
    bv.band_ids = b.band;
    bv.schema_allow = b.has_rule ? b.sa : nullptr;
    bv.band_allow = b.has_rule ? b.ba : nullptr;
    kc_batch_out out{};
    out.p = b.p;
    out.p_capacity = s->max_p;
    out.index = b.index;
    out.q_capacity = s->max_records;
    out.p_off = b.p_off;
    out.q_off = b.q_off;
    kc_status st;
    std::string err;
    {
      std::lock_guard<std::mutex> hl(s->h->mu);
      DeviceGuard dg(s->h->device);
      st = forward_batch_host(s->h, &bv, &out);
      if (st) err = s->h->err;
    }
    {
      std::lock_guard<std::mutex> lk(s->mu);
      b.status = st;
      b.err = err;
      b.done_ms = steady_ms();
      b.state = kDone;
      s->queue.erase(std::find(s->queue.begin(), s->queue.end(), idx));
      s->done.push_back(idx);
    }
    s->cv.notify_all();
  }
}

// The open buffer, opening a free one if none is open. -1 if every buffer is
// sealed, running, done or handed out.
int open_buffer(kc_stream* s) {
  if (s->open >= 0) return s->open;
  for (size_t i = 0; i < s->bufs.size(); i++)
    if (s->bufs[i].state == kFree) {
      StreamBuf& b = s->bufs[i];
      b.state = kOpen;
      b.frames = 0;
      b.records = b.questions = b.p_total = 0;
      b.has_rule = false;
      b.rec_off[0] = 0;
      b.first_ticket = s->next_ticket;
      s->open = int(i);
      return s->open;
    }
  return -1;
}

}  // namespace

extern "C" {

kc_status kc_stream_create(kc_handle* h, uint32_t max_frames, uint64_t max_records, uint64_t max_p, uint32_t depth,
                           kc_stream** out) {
  if (!h) return fail(nullptr, KC_ERR_INVALID_ARG, "handle is null");
  if (!out) return fail(h, KC_ERR_INVALID_ARG, "out is null");
  *out = nullptr;
  if (max_frames == 0 || max_records == 0 || depth < 2)
    return fail(h, KC_ERR_INVALID_ARG, "a stream needs room for a frame, a record and at least two buffers");
  auto* s = new kc_stream();
  s->h = h;
  s->max_frames = max_frames;
  s->max_records = max_records;
  s->max_p = max_p ? max_p : max_records * 64;
  s->bufs.resize(depth);
  DeviceGuard dg(h->device);
  for (StreamBuf& b : s->bufs) {
    cudaError_t e = cudaSuccess;
    auto host = [&](void** p, size_t bytes) {
      if (e == cudaSuccess) e = cudaMallocHost(p, bytes ? bytes : 16);
    };
    host(reinterpret_cast<void**>(&b.rec_off), (max_frames + 1ull) * 8);
    host(reinterpret_cast<void**>(&b.tok), max_records * 32);
    host(reinterpret_cast<void**>(&b.role), max_records * 32);
    host(reinterpret_cast<void**>(&b.sch), max_records * 4);
    host(reinterpret_cast<void**>(&b.band), max_records * 4);
    host(reinterpret_cast<void**>(&b.sa), max_records * 32);
    host(reinterpret_cast<void**>(&b.ba), max_records * 4);
    host(reinterpret_cast<void**>(&b.p), s->max_p * 4);
    host(reinterpret_cast<void**>(&b.index), max_records * 4);
    host(reinterpret_cast<void**>(&b.p_off), (max_frames + 1ull) * 8);
    host(reinterpret_cast<void**>(&b.q_off), (max_frames + 1ull) * 8);
    if (e != cudaSuccess) {
      for (StreamBuf& x : s->bufs) free_buf(x);
      delete s;
      return cuda_fail(h, e, "stream staging");
    }
  }
  s->worker = std::thread(stream_worker, s);
  *out = s;
  return KC_OK;
}

kc_status kc_stream_push(kc_stream* s, const kc_frame_view* frame, const uint32_t* schema_allow,
                         const uint32_t* band_allow, uint64_t* ticket) {
  if (!s) return KC_ERR_INVALID_ARG;
  if (!frame || !frame->token_ids || !frame->field_roles || !frame->schema_ids || !frame->band_ids)
    return stream_fail(s, KC_ERR_INVALID_ARG, "frame view is incomplete");
  if ((schema_allow == nullptr) != (band_allow == nullptr))
    return stream_fail(s, KC_ERR_INVALID_ARG, "a mask rule needs both schema_allow and band_allow");
  const kc_handle* h = s->h;
  const Dims& d = h->d;
  // compileActiveFrame's walk: the active list in order, to the first unoccupied entry
  const uint32_t slots = frame->slots;
  thread_local std::vector<uint32_t> act;
  act.clear();
  for (uint32_t i = 0; i < slots; i++) {
    const uint32_t a = frame->active_record_indices ? frame->active_record_indices[i] : i;
    if (a == KC_INVALID || a >= slots) break;
    act.push_back(a);
  }
  const uint64_t n = act.size();
  if (n == 0) return stream_fail(s, KC_ERR_INVALID_ARG, "a frame with no records has nothing to think about");
  // the batch path's validation, on the host, before the frame joins a batch:
  // one table lookup per token id and role id (bit 0: a valid token, bit 1: a
  // valid field role); the precise refusal is worked out only on failure
  const uint8_t* ok = h->id_ok.data();
  const uint32_t len = h->token_rows_len;
  uint64_t q = 0;
  bool bad = false;
  for (uint32_t a : act) {
    const uint32_t* ids = frame->token_ids + a * 8ull;
    const uint32_t* roles = frame->field_roles + a * 8ull;
    for (int l = 0; l < 8; l++) {
      const uint32_t id = ids[l], role = roles[l];
      const uint32_t ft = id < len ? ok[id] : 0u, fr = role < len ? ok[role] : 0u;
      bad |= id != 0 && !((ft & 1u) && (fr & 2u));
    }
    bad |= frame->schema_ids[a] >= d.schema_space || frame->band_ids[a] >= d.band_space;
    q += frame->band_ids[a] == KC_QUERY_BAND;
  }
  if (bad) {
    for (uint32_t a : act) {
      for (int l = 0; l < 8; l++) {
        const uint32_t id = frame->token_ids[a * 8ull + l];
        if (id == 0) continue;
        const uint32_t role = frame->field_roles[a * 8ull + l];
        if (id >= len) return stream_fail(s, KC_ERR_INVALID_ARG, "token id has no entry in tokenRows");
        if (h->token_rows_host[id] >= d.token_space)
          return stream_fail(s, KC_ERR_INVALID_ARG, "token row outside the token table");
        if (role >= len) return stream_fail(s, KC_ERR_INVALID_ARG, "field role id has no entry in tokenRows");
        if (h->token_rows_host[role] >= d.field_space)
          return stream_fail(s, KC_ERR_INVALID_ARG, "field role row outside the field table");
      }
      if (frame->schema_ids[a] >= d.schema_space)
        return stream_fail(s, KC_ERR_INVALID_ARG, "schema id outside the schema table");
      if (frame->band_ids[a] >= d.band_space)
        return stream_fail(s, KC_ERR_INVALID_ARG, "band id outside the band table");
    }
  }
  const uint64_t r = n - q;
  if (r > KC_MAX_BANK) return stream_fail(s, KC_ERR_CAPACITY, "bank records exceed capacity");
  if (n > s->max_records || q * r > s->max_p)
    return stream_fail(s, KC_ERR_CAPACITY, "the frame is larger than a stream buffer");
  std::lock_guard<std::mutex> lk(s->mu);
  int bi = open_buffer(s);
  if (bi < 0) return stream_fail(s, KC_ERR_CAPACITY, "every stream buffer is in flight or unpolled: poll first");
  StreamBuf* b = &s->bufs[bi];
  if (b->frames + 1 > s->max_frames || b->records + n > s->max_records || b->p_total + q * r > s->max_p)
    return stream_fail(s, KC_ERR_CAPACITY, "the open stream buffer is full: flush first");
  const uint64_t r0 = b->records;
  for (uint64_t i = 0; i < n; i++) {
    const uint32_t a = act[i];
    memcpy(b->tok + (r0 + i) * 8, frame->token_ids + a * 8ull, 32);
    memcpy(b->role + (r0 + i) * 8, frame->field_roles + a * 8ull, 32);
    b->sch[r0 + i] = frame->schema_ids[a];
    b->band[r0 + i] = frame->band_ids[a];
  }
  if (schema_allow && !b->has_rule) {  // earlier questions of this buffer admit everything
    for (uint64_t i = 0; i < b->questions * 8; i++) b->sa[i] = 0xffffffffu;
    for (uint64_t i = 0; i < b->questions; i++) b->ba[i] = 0xffffffffu;
    b->has_rule = true;
  }
  if (b->has_rule) {
    for (uint64_t i = 0; i < q; i++) {
      for (int w = 0; w < 8; w++) b->sa[(b->questions + i) * 8 + w] = schema_allow ? schema_allow[i * 8 + w] : 0xffffffffu;
      b->ba[b->questions + i] = band_allow ? band_allow[i] : 0xffffffffu;
    }
  }
  b->records += n;
  b->questions += q;
  b->p_total += q * r;
  b->frames++;
  b->rec_off[b->frames] = b->records;
  if (ticket) *ticket = s->next_ticket;
  s->next_ticket++;
  return KC_OK;
}

kc_status kc_stream_push_many(kc_stream* s, const kc_batch_view* frames, uint64_t* first_ticket, uint32_t* pushed) {
  if (!s) return KC_ERR_INVALID_ARG;
  if (pushed) *pushed = 0;
  if (!frames || !frames->rec_off) return stream_fail(s, KC_ERR_INVALID_ARG, "batch view is incomplete");
  if ((frames->schema_allow == nullptr) != (frames->band_allow == nullptr))
    return stream_fail(s, KC_ERR_INVALID_ARG, "a mask rule needs both schema_allow and band_allow");
  uint64_t q_seen = 0;  // questions of the frames before this one (indexes the rule)
  for (uint32_t f = 0; f < frames->frames; f++) {
    const uint64_t r0 = frames->rec_off[f], r1 = frames->rec_off[f + 1];
    if (r1 < r0) return stream_fail(s, KC_ERR_INVALID_ARG, "rec_off must not decrease");
    kc_frame_view v{};
    v.slots = uint32_t(r1 - r0);
    v.token_ids = frames->token_ids + r0 * 8;
    v.field_roles = frames->field_roles + r0 * 8;
    v.schema_ids = frames->schema_ids + r0;
    v.band_ids = frames->band_ids + r0;
    v.active_record_indices = nullptr;  // every record active, in order
    uint64_t q = 0;
    for (uint64_t g = r0; g < r1; g++) q += frames->band_ids[g] == KC_QUERY_BAND;
    const uint32_t* sa = frames->schema_allow ? frames->schema_allow + q_seen * 8 : nullptr;
    const uint32_t* ba = frames->band_allow ? frames->band_allow + q_seen : nullptr;
    uint64_t t = 0;
    const kc_status st = kc_stream_push(s, &v, sa, ba, &t);
    if (st) return st;
    if (f == 0 && first_ticket) *first_ticket = t;
    if (pushed) *pushed = f + 1;
    q_seen += q;
  }
  return KC_OK;
}

kc_status kc_stream_flush(kc_stream* s) {
  if (!s) return KC_ERR_INVALID_ARG;
  {
    std::lock_guard<std::mutex> lk(s->mu);
    if (s->open < 0 || s->bufs[s->open].frames == 0) return KC_OK;
    StreamBuf& b = s->bufs[s->open];
    b.state = kSealed;
    b.seal_ms = steady_ms();
    s->queue.push_back(s->open);
    s->open = -1;
  }
  s->cv.notify_all();
  return KC_OK;
}

uint32_t kc_stream_pending(kc_stream* s) {
  if (!s) return 0;
  std::lock_guard<std::mutex> lk(s->mu);
  return uint32_t(s->queue.size());
}

kc_status kc_stream_poll(kc_stream* s, int wait, kc_stream_result* out) {
  if (!s || !out) return KC_ERR_INVALID_ARG;
  std::unique_lock<std::mutex> lk(s->mu);
  if (s->handed >= 0) {  // the batch handed out last time is released
    s->bufs[s->handed].state = kFree;
    s->handed = -1;
  }
  *out = kc_stream_result{};
  if (wait) s->cv.wait(lk, [&] { return !s->done.empty() || s->queue.empty(); });
  if (s->done.empty()) return KC_OK;
  const int i = s->done.front();
  s->done.pop_front();
  StreamBuf& b = s->bufs[i];
  b.state = kHanded;
  s->handed = i;
  out->first_ticket = b.first_ticket;
  out->frames = b.frames;
  out->questions = b.questions;
  out->total_p = b.p_total;
  out->p_off = b.p_off;
  out->q_off = b.q_off;
  out->p = b.p;
  out->index = b.index;
  out->status = b.status;
  out->error = b.status ? b.err.c_str() : nullptr;
  out->sealed_ms = b.seal_ms;
  out->done_ms = b.done_ms;
  return KC_OK;
}

double kc_stream_clock_ms(void) { return steady_ms(); }

const char* kc_stream_last_error(kc_stream* s) { return s ? s->err.c_str() : ""; }

void kc_stream_destroy(kc_stream* s) {
  if (!s) return;
  {
    std::unique_lock<std::mutex> lk(s->mu);
    s->cv.wait(lk, [&] {  // let queued batches finish: the worker may be inside one
      for (int i : s->queue)
        if (s->bufs[i].state == kRunning) return false;
      return true;
    });
    s->stop = true;
  }
  s->cv.notify_all();
  if (s->worker.joinable()) s->worker.join();
  for (StreamBuf& b : s->bufs) free_buf(b);
  delete s;
}

}  // extern "C"
