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
//          failing the batch it would have joined; push_many does the same
//          for a run of frames, the validation and copies split over helper
//          threads;
//   flush  seals the open buffer and queues it; a worker thread runs sealed
//          buffers back to back through the batch path (H2D from pinned
//          memory, GPU packing, encode, select, D2H into the buffer's pinned
//          result arrays), while the caller keeps pushing into the next
//          buffer;
//   poll   hands back the oldest finished batch: its ticket range, per-frame
//          offsets, p and indices, and the steady-clock times at which it was
//          sealed, started and finished.
//
// Buffers cycle free -> open -> sealed -> running -> done -> handed out; the
// batch handed out by a poll stays readable until the next poll.
//
// Placement. The host side of a batch is two streams of memory traffic: the
// pushes write every record into the staging (72 bytes a record), and the
// copy engines read the staging and write the results back over PCIe. When
// the staging pages, the worker or the pushing threads sit on the other CPU
// socket than the GPU, both cross the socket link and the worker's waits
// compete with whatever else runs there, so that the same program ran at
// very different rates from one launch to the next. With binding on (the
// default), the worker and the helper threads run on the CPUs that sysfs
// lists as local to the GPU (intersected with the CPUs this process may use),
// and the worker allocates the staging, so that its pages are placed on the
// GPU's node. kc_stream_read_stats reports where everything landed and where
// the host time went.

#include <atomic>
#include <cctype>
#include <condition_variable>
#include <deque>
#include <fstream>
#include <functional>
#include <thread>

#include <pthread.h>
#include <sched.h>
#include <sys/resource.h>
#include <sys/syscall.h>
#include <unistd.h>

namespace {

double steady_ms() { return now_ms(); }

enum BufState { kFree = 0, kOpen, kSealed, kRunning, kDone, kHanded };

// push_many calls over fewer records than this run on the caller alone: the
// helpers' wake-up costs more than they would save
constexpr uint64_t kParallelPushRecords = 16384;

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
  double seal_ms = 0, start_ms = 0, done_ms = 0, wait_ms = 0;
};

// ---- placement ------------------------------------------------------------

// The CPUs of a sysfs cpulist ("0-55,112-167"); empty when unreadable.
std::vector<int> read_cpulist(const std::string& path) {
  std::ifstream f(path);
  std::string line;
  std::vector<int> out;
  if (!f || !std::getline(f, line)) return out;
  size_t i = 0;
  while (i < line.size()) {
    size_t j = line.find(',', i);
    if (j == std::string::npos) j = line.size();
    const std::string part = line.substr(i, j - i);
    i = j + 1;
    if (part.empty() || !isdigit(static_cast<unsigned char>(part[0]))) continue;
    const int a = atoi(part.c_str());
    const size_t dash = part.find('-');
    const int b = dash == std::string::npos ? a : atoi(part.c_str() + dash + 1);
    for (int c = a; c <= b && c < CPU_SETSIZE; c++) out.push_back(c);
  }
  return out;
}

struct GpuPlacement {
  int node = -1;          // the GPU's NUMA node (sysfs numa_node), -1 unknown
  std::vector<int> cpus;  // CPUs local to the GPU that this process may run on
};

GpuPlacement gpu_placement(int device) {
  GpuPlacement g;
  char bus[64] = {0};
  if (cudaDeviceGetPCIBusId(bus, sizeof bus, device) != cudaSuccess) return g;
  unsigned dom = 0, b = 0, dev = 0, fn = 0;
  if (sscanf(bus, "%x:%x:%x.%x", &dom, &b, &dev, &fn) != 4) return g;
  char id[32];
  snprintf(id, sizeof id, "%04x:%02x:%02x.%x", dom & 0xffffu, b, dev, fn);
  const std::string dir = std::string("/sys/bus/pci/devices/") + id + "/";
  {
    std::ifstream f(dir + "numa_node");
    int n = -1;
    if (f >> n) g.node = n;
  }
  cpu_set_t allowed;
  CPU_ZERO(&allowed);
  if (sched_getaffinity(0, sizeof allowed, &allowed) != 0) return g;
  for (int c : read_cpulist(dir + "local_cpulist"))
    if (CPU_ISSET(c, &allowed)) g.cpus.push_back(c);
  return g;
}

bool bind_self(const std::vector<int>& cpus) {
  if (cpus.empty()) return false;
  cpu_set_t set;
  CPU_ZERO(&set);
  for (int c : cpus) CPU_SET(c, &set);
  return pthread_setaffinity_np(pthread_self(), sizeof set, &set) == 0;
}

// The calling thread's CPU and NUMA node (-1 when the kernel does not say).
void where_am_i(int* cpu, int* node) {
  unsigned c = 0, n = 0;
  if (syscall(SYS_getcpu, &c, &n, nullptr) == 0) {
    *cpu = int(c);
    *node = int(n);
  } else {
    *cpu = *node = -1;
  }
}

// The NUMA node of the page holding p (move_pages asked for nodes only).
int page_node(const void* p) {
  void* pages[1] = {const_cast<void*>(p)};
  int status[1] = {-1};
  if (syscall(SYS_move_pages, 0, 1ul, pages, nullptr, status, 0) != 0) return -1;
  return status[0] >= 0 ? status[0] : -1;
}

struct ThreadUsage {
  uint64_t minflt = 0, majflt = 0, nvcsw = 0, nivcsw = 0;
};

ThreadUsage thread_usage() {
  rusage r{};
  ThreadUsage u;
  if (getrusage(RUSAGE_THREAD, &r) == 0) {
    u.minflt = uint64_t(r.ru_minflt);
    u.majflt = uint64_t(r.ru_majflt);
    u.nvcsw = uint64_t(r.ru_nvcsw);
    u.nivcsw = uint64_t(r.ru_nivcsw);
  }
  return u;
}

// ---- helper threads for push_many ------------------------------------------

// run(n, f) calls f(0) on the caller and f(1) .. f(n-1) on helpers, and
// returns when all n have returned.
struct PushPool {
  std::vector<std::thread> threads;
  std::mutex mu;
  std::condition_variable go, done;
  const std::function<void(int)>* job = nullptr;
  int parts = 0, remaining = 0;
  uint64_t gen = 0;
  bool stop = false;

  void start(int helpers, const std::vector<int>& cpus) {
    for (int i = 0; i < helpers; i++)
      threads.emplace_back([this, i, cpus] {
        bind_self(cpus);
        uint64_t seen = 0;
        for (;;) {
          const std::function<void(int)>* j;
          const int part = i + 1;
          {
            std::unique_lock<std::mutex> lk(mu);
            go.wait(lk, [&] { return stop || gen != seen; });
            if (stop) return;
            seen = gen;
            if (part >= parts) continue;
            j = job;
          }
          (*j)(part);
          {
            std::lock_guard<std::mutex> lk(mu);
            if (--remaining == 0) done.notify_all();
          }
        }
      });
  }
  int size() const { return int(threads.size()) + 1; }
  void run(int n, const std::function<void(int)>& f) {
    n = std::max(1, std::min(n, size()));
    if (n > 1) {
      {
        std::lock_guard<std::mutex> lk(mu);
        job = &f;
        parts = n;
        remaining = n - 1;
        gen++;
      }
      go.notify_all();
    }
    f(0);
    if (n > 1) {
      std::unique_lock<std::mutex> lk(mu);
      done.wait(lk, [&] { return remaining == 0; });
      job = nullptr;
    }
  }
  void shut() {
    {
      std::lock_guard<std::mutex> lk(mu);
      stop = true;
    }
    go.notify_all();
    for (std::thread& t : threads)
      if (t.joinable()) t.join();
    threads.clear();
  }
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
  // mu guards the buffer states, the queues and the worker's statistics;
  // push_mu serialises the pushes and flushes that fill the open buffer
  // (taken before mu), so that the worker never waits for a push's copies
  std::mutex mu, push_mu;
  std::condition_variable cv;
  std::thread worker;
  int ready = 0;  // the worker's start-up: 1 staging allocated, -1 failed
  cudaError_t alloc_err = cudaSuccess;
  bool stop = false;
  std::string err;
  // placement and helpers
  bool bind = true;
  GpuPlacement place;
  PushPool pool;
  std::vector<uint32_t> frame_q;   // push_many: questions per frame
  std::vector<uint8_t> frame_bad;  // push_many: a frame that failed the id checks
  kc_stream_stats stats{};
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
  b = StreamBuf{};
}

cudaError_t alloc_buf(kc_stream* s, StreamBuf& b) {
  cudaError_t e = cudaSuccess;
  auto host = [&](void** p, size_t bytes) {
    if (e == cudaSuccess) e = cudaMallocHost(p, bytes ? bytes : 16);
  };
  const uint64_t mr = s->max_records;
  host(reinterpret_cast<void**>(&b.rec_off), (s->max_frames + 1ull) * 8);
  host(reinterpret_cast<void**>(&b.tok), mr * 32);
  host(reinterpret_cast<void**>(&b.role), mr * 32);
  host(reinterpret_cast<void**>(&b.sch), mr * 4);
  host(reinterpret_cast<void**>(&b.band), mr * 4);
  host(reinterpret_cast<void**>(&b.sa), mr * 32);
  host(reinterpret_cast<void**>(&b.ba), mr * 4);
  host(reinterpret_cast<void**>(&b.p), s->max_p * 4);
  host(reinterpret_cast<void**>(&b.index), mr * 4);
  host(reinterpret_cast<void**>(&b.p_off), (s->max_frames + 1ull) * 8);
  host(reinterpret_cast<void**>(&b.q_off), (s->max_frames + 1ull) * 8);
  return e;
}

// The worker: allocates the staging (on the GPU's node when bound), then runs
// sealed buffers in order through the batch path.
void stream_worker(kc_stream* s) {
  cudaSetDevice(s->h->device);
  const bool bound = s->bind && bind_self(s->place.cpus);
  cudaError_t e = cudaSuccess;
  for (StreamBuf& b : s->bufs)
    if (e == cudaSuccess) e = alloc_buf(s, b);
  {
    std::lock_guard<std::mutex> lk(s->mu);
    s->alloc_err = e;
    s->ready = e == cudaSuccess ? 1 : -1;
    s->stats.bound_cpus = bound ? uint32_t(s->place.cpus.size()) : 0;
    s->stats.staging_numa_node = e == cudaSuccess ? page_node(s->bufs[0].tok) : -1;
  }
  s->cv.notify_all();
  if (e != cudaSuccess) return;
  for (;;) {
    int idx;
    const double idle0 = steady_ms();
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
      s->stats.idle_ms += steady_ms() - idle0;
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
    int cpu0, node0, cpu1, node1;
    where_am_i(&cpu0, &node0);
    const ThreadUsage u0 = thread_usage();
    const uint64_t g0 = t_grows;
    const double gms0 = t_grow_ms;
    const double t0 = steady_ms();
    double waited;
    {
      std::lock_guard<std::mutex> hl(s->h->mu);
      DeviceGuard dg(s->h->device);
      const double w0 = s->h->host_wait_ms;
      st = forward_batch_host(s->h, &bv, &out);
      waited = s->h->host_wait_ms - w0;
      if (st) err = s->h->err;
    }
    const double t1 = steady_ms();
    const ThreadUsage u1 = thread_usage();
    where_am_i(&cpu1, &node1);
    {
      std::lock_guard<std::mutex> lk(s->mu);
      b.status = st;
      b.err = err;
      b.start_ms = t0;
      b.done_ms = t1;
      b.wait_ms = waited;
      b.state = kDone;
      s->queue.erase(std::find(s->queue.begin(), s->queue.end(), idx));
      s->done.push_back(idx);
      kc_stream_stats& x = s->stats;
      x.batches++;
      x.run_ms += t1 - t0;
      x.sync_wait_ms += waited;
      x.workspace_grows += t_grows - g0;
      x.workspace_grow_ms += t_grow_ms - gms0;
      x.worker_minor_faults += u1.minflt - u0.minflt;
      x.worker_major_faults += u1.majflt - u0.majflt;
      x.worker_voluntary_switches += u1.nvcsw - u0.nvcsw;
      x.worker_involuntary_switches += u1.nivcsw - u0.nivcsw;
      x.worker_cpu_moves += cpu0 != cpu1;
      x.worker_numa_node = node1;
    }
    s->cv.notify_all();
  }
}

// The open buffer, opening a free one if none is open. -1 if every buffer is
// sealed, running, done or handed out. Called with s->mu held.
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

int open_buffer_locked(kc_stream* s) {
  std::lock_guard<std::mutex> lk(s->mu);
  return open_buffer(s);
}

// The id and table checks of one frame's records (the batch path's
// validation, done on the host before the frame joins a batch): one table
// lookup per token id and role id (bit 0: a valid token, bit 1: a valid field
// role). Counts the frame's questions into *q. False if any record fails.
bool frame_ids_ok(const kc_handle* h, const uint32_t* tok, const uint32_t* role, const uint32_t* sch,
                  const uint32_t* band, const uint32_t* act, uint64_t n, uint64_t* q) {
  const Dims& d = h->d;
  const uint8_t* ok = h->id_ok.data();
  const uint32_t len = h->token_rows_len;
  bool bad = false;
  uint64_t nq = 0;
  for (uint64_t i = 0; i < n; i++) {
    const uint64_t a = act ? act[i] : i;
    const uint32_t* ids = tok + a * 8;
    const uint32_t* roles = role + a * 8;
    for (int l = 0; l < 8; l++) {
      const uint32_t id = ids[l], r = roles[l];
      const uint32_t ft = id < len ? ok[id] : 0u, fr = r < len ? ok[r] : 0u;
      bad |= id != 0 && !((ft & 1u) && (fr & 2u));
    }
    bad |= sch[a] >= d.schema_space || band[a] >= d.band_space;
    nq += band[a] == KC_QUERY_BAND;
  }
  *q = nq;
  return !bad;
}

// The precise refusal of a frame that failed frame_ids_ok.
kc_status frame_refusal(kc_stream* s, const uint32_t* tok, const uint32_t* role, const uint32_t* sch,
                        const uint32_t* band, const uint32_t* act, uint64_t n) {
  const kc_handle* h = s->h;
  const Dims& d = h->d;
  const uint32_t len = h->token_rows_len;
  for (uint64_t i = 0; i < n; i++) {
    const uint64_t a = act ? act[i] : i;
    for (int l = 0; l < 8; l++) {
      const uint32_t id = tok[a * 8 + l];
      if (id == 0) continue;
      const uint32_t r = role[a * 8 + l];
      if (id >= len) return stream_fail(s, KC_ERR_INVALID_ARG, "token id has no entry in tokenRows");
      if (h->token_rows_host[id] >= d.token_space)
        return stream_fail(s, KC_ERR_INVALID_ARG, "token row outside the token table");
      if (r >= len) return stream_fail(s, KC_ERR_INVALID_ARG, "field role id has no entry in tokenRows");
      if (h->token_rows_host[r] >= d.field_space)
        return stream_fail(s, KC_ERR_INVALID_ARG, "field role row outside the field table");
    }
    if (sch[a] >= d.schema_space) return stream_fail(s, KC_ERR_INVALID_ARG, "schema id outside the schema table");
    if (band[a] >= d.band_space) return stream_fail(s, KC_ERR_INVALID_ARG, "band id outside the band table");
  }
  return stream_fail(s, KC_ERR_INVALID_ARG, "frame failed validation");
}

// A frame's place in the open buffer: the capacity checks of one frame of n
// records and q questions, in the order a single push makes them. KC_OK with
// *bi the open buffer, or the refusal.
kc_status frame_fits(kc_stream* s, uint64_t n, uint64_t q, uint32_t frames_before, uint64_t records_before,
                     uint64_t p_before, bool may_open, int* bi) {
  const uint64_t r = n - q;
  if (r > KC_MAX_BANK) return stream_fail(s, KC_ERR_CAPACITY, "bank records exceed capacity");
  if (n > s->max_records || q * r > s->max_p)
    return stream_fail(s, KC_ERR_CAPACITY, "the frame is larger than a stream buffer");
  if (*bi < 0 && may_open) *bi = open_buffer_locked(s);
  if (*bi < 0) return stream_fail(s, KC_ERR_CAPACITY, "every stream buffer is in flight or unpolled: poll first");
  const StreamBuf& b = s->bufs[*bi];
  if (b.frames + frames_before + 1 > s->max_frames || b.records + records_before + n > s->max_records ||
      b.p_total + p_before + q * r > s->max_p)
    return stream_fail(s, KC_ERR_CAPACITY, "the open stream buffer is full: flush first");
  return KC_OK;
}

// Writes questions q0 .. q0+nq-1 of the buffer's rule: the given rows, or the
// open rule (everything admitted) when none is given.
void write_rule(StreamBuf* b, uint64_t q0, uint64_t nq, const uint32_t* sa, const uint32_t* ba) {
  if (sa) {
    memcpy(b->sa + q0 * 8, sa, nq * 32);
    memcpy(b->ba + q0, ba, nq * 4);
  } else {
    std::fill(b->sa + q0 * 8, b->sa + (q0 + nq) * 8, 0xffffffffu);
    std::fill(b->ba + q0, b->ba + q0 + nq, 0xffffffffu);
  }
}

// A buffer takes a rule for the first time: its earlier questions admit
// everything.
void open_rule(StreamBuf* b) {
  if (b->has_rule) return;
  write_rule(b, 0, b->questions, nullptr, nullptr);
  b->has_rule = true;
}

}  // namespace

extern "C" {

kc_status kc_stream_create_ex(kc_handle* h, uint32_t max_frames, uint64_t max_records, uint64_t max_p,
                              uint32_t depth, const kc_stream_options* opts, kc_stream** out) {
  if (!h) return fail(nullptr, KC_ERR_INVALID_ARG, "handle is null");
  if (!out) return fail(h, KC_ERR_INVALID_ARG, "out is null");
  *out = nullptr;
  if (max_frames == 0 || max_records == 0 || depth < 2)
    return fail(h, KC_ERR_INVALID_ARG, "a stream needs room for a frame, a record and at least two buffers");
  kc_stream_options o{0, 1};
  if (opts) o = *opts;
  auto* s = new kc_stream();
  s->h = h;
  s->max_frames = max_frames;
  s->max_records = max_records;
  s->max_p = max_p ? max_p : max_records * 64;
  s->bufs.resize(depth);
  s->bind = o.bind_cpus != 0;
  s->place = gpu_placement(h->device);
  s->stats.gpu_numa_node = s->place.node;
  s->stats.staging_numa_node = s->stats.worker_numa_node = s->stats.caller_numa_node = -1;
  int threads = int(o.push_threads);
  if (threads == 0) threads = std::max(1, std::min(8, int(s->place.cpus.size()) / 4));
  threads = std::max(1, std::min(threads, 64));
  s->stats.push_threads = uint32_t(threads);
  s->worker = std::thread(stream_worker, s);
  {
    std::unique_lock<std::mutex> lk(s->mu);
    s->cv.wait(lk, [&] { return s->ready != 0; });
  }
  if (s->ready < 0) {
    s->worker.join();
    const cudaError_t e = s->alloc_err;
    for (StreamBuf& b : s->bufs) free_buf(b);
    delete s;
    return cuda_fail(h, e, "stream staging");
  }
  s->pool.start(threads - 1, s->bind ? s->place.cpus : std::vector<int>{});
  *out = s;
  return KC_OK;
}

kc_status kc_stream_create(kc_handle* h, uint32_t max_frames, uint64_t max_records, uint64_t max_p, uint32_t depth,
                           kc_stream** out) {
  return kc_stream_create_ex(h, max_frames, max_records, max_p, depth, nullptr, out);
}

kc_status kc_stream_push(kc_stream* s, const kc_frame_view* frame, const uint32_t* schema_allow,
                         const uint32_t* band_allow, uint64_t* ticket) {
  if (!s) return KC_ERR_INVALID_ARG;
  if (!frame || !frame->token_ids || !frame->field_roles || !frame->schema_ids || !frame->band_ids)
    return stream_fail(s, KC_ERR_INVALID_ARG, "frame view is incomplete");
  if ((schema_allow == nullptr) != (band_allow == nullptr))
    return stream_fail(s, KC_ERR_INVALID_ARG, "a mask rule needs both schema_allow and band_allow");
  const double t0 = steady_ms();
  std::lock_guard<std::mutex> pl(s->push_mu);
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
  uint64_t q = 0;
  if (!frame_ids_ok(s->h, frame->token_ids, frame->field_roles, frame->schema_ids, frame->band_ids, act.data(), n, &q))
    return frame_refusal(s, frame->token_ids, frame->field_roles, frame->schema_ids, frame->band_ids, act.data(), n);
  int bi = s->open;
  kc_status st = frame_fits(s, n, q, 0, 0, 0, true, &bi);
  if (st) return st;
  StreamBuf* b = &s->bufs[bi];
  const uint64_t r0 = b->records;
  for (uint64_t i = 0; i < n; i++) {
    const uint32_t a = act[i];
    memcpy(b->tok + (r0 + i) * 8, frame->token_ids + a * 8ull, 32);
    memcpy(b->role + (r0 + i) * 8, frame->field_roles + a * 8ull, 32);
    b->sch[r0 + i] = frame->schema_ids[a];
    b->band[r0 + i] = frame->band_ids[a];
  }
  if (schema_allow) open_rule(b);
  if (b->has_rule) write_rule(b, b->questions, q, schema_allow, band_allow);
  b->records += n;
  b->questions += q;
  b->p_total += q * (n - q);
  b->frames++;
  b->rec_off[b->frames] = b->records;
  if (ticket) *ticket = s->next_ticket;
  s->next_ticket++;
  s->stats.push_calls++;
  s->stats.frames_pushed++;
  s->stats.bytes_staged += n * 72 + (b->has_rule ? q * 36 : 0);
  s->stats.push_ms += steady_ms() - t0;
  return KC_OK;
}

kc_status kc_stream_push_many(kc_stream* s, const kc_batch_view* frames, uint64_t* first_ticket, uint32_t* pushed) {
  if (!s) return KC_ERR_INVALID_ARG;
  if (pushed) *pushed = 0;
  if (!frames || !frames->rec_off) return stream_fail(s, KC_ERR_INVALID_ARG, "batch view is incomplete");
  if ((frames->schema_allow == nullptr) != (frames->band_allow == nullptr))
    return stream_fail(s, KC_ERR_INVALID_ARG, "a mask rule needs both schema_allow and band_allow");
  const uint32_t F = frames->frames;
  if (F == 0) return KC_OK;
  if (!frames->token_ids || !frames->field_roles || !frames->schema_ids || !frames->band_ids)
    return stream_fail(s, KC_ERR_INVALID_ARG, "frame view is incomplete");
  const double t0 = steady_ms();
  const ThreadUsage u0 = thread_usage();
  std::lock_guard<std::mutex> pl(s->push_mu);
  const uint64_t* ro = frames->rec_off;
  // frames up to the first whose offsets run backwards are looked at
  uint32_t lim = 0;
  while (lim < F && ro[lim + 1] >= ro[lim]) lim++;
  // 1. every frame's questions and id checks, and its records copied to where
  //    they land if every frame before it is taken (the frames taken are a
  //    prefix, and their records are one run of the source and of the
  //    staging); a frame past the staging's room is only checked
  int bi = s->open;
  if (bi < 0) bi = open_buffer_locked(s);  // -1: refused below, after the first frame's checks
  StreamBuf* b = bi >= 0 ? &s->bufs[bi] : nullptr;
  const uint64_t rec_room = b ? s->max_records - b->records : 0;
  s->frame_q.resize(lim);
  s->frame_bad.resize(lim);
  const uint64_t total = ro[lim] - ro[0];
  const int parts = total >= kParallelPushRecords ? s->pool.size() : 1;
  const std::function<void(int)> pass = [&](int part) {
    // frames of this part: an equal share of the records
    const uint64_t lo = ro[0] + total * uint64_t(part) / uint64_t(parts);
    const uint64_t hi = ro[0] + total * uint64_t(part + 1) / uint64_t(parts);
    // a frame belongs to the part where it starts (ro is sorted up to lim)
    uint32_t f = uint32_t(std::lower_bound(ro, ro + lim, lo) - ro);
    for (; f < lim && (ro[f] < hi || part == parts - 1); f++) {
      const uint64_t n = ro[f + 1] - ro[f];
      uint64_t q = 0;
      s->frame_bad[f] = !frame_ids_ok(s->h, frames->token_ids + ro[f] * 8, frames->field_roles + ro[f] * 8,
                                      frames->schema_ids + ro[f], frames->band_ids + ro[f], nullptr, n, &q);
      s->frame_q[f] = uint32_t(q);
      const uint64_t d = ro[f] - ro[0];  // the frame's first record in this call's run
      if (b && d + n <= rec_room) {
        const uint64_t at = b->records + d;
        memcpy(b->tok + at * 8, frames->token_ids + ro[f] * 8, n * 32);
        memcpy(b->role + at * 8, frames->field_roles + ro[f] * 8, n * 32);
        memcpy(b->sch + at, frames->schema_ids + ro[f], n * 4);
        memcpy(b->band + at, frames->band_ids + ro[f], n * 4);
      }
    }
  };
  s->pool.run(parts, pass);
  // 2. the frames taken, in order, with the refusals a frame-by-frame push
  //    would give
  kc_status st = KC_OK;
  uint32_t k = 0;
  uint64_t recs = 0, qs = 0, ps = 0;
  for (; k < lim; k++) {
    const uint64_t n = ro[k + 1] - ro[k], q = s->frame_q[k];
    if (n == 0) {
      st = stream_fail(s, KC_ERR_INVALID_ARG, "a frame with no records has nothing to think about");
      break;
    }
    if (s->frame_bad[k]) {
      st = frame_refusal(s, frames->token_ids + ro[k] * 8, frames->field_roles + ro[k] * 8,
                         frames->schema_ids + ro[k], frames->band_ids + ro[k], nullptr, n);
      break;
    }
    if ((st = frame_fits(s, n, q, k, recs, ps, false, &bi))) break;  // only the buffer the pass filled
    recs += n;
    qs += q;
    ps += q * (n - q);
  }
  if (!st && lim < F) st = stream_fail(s, KC_ERR_INVALID_ARG, "rec_off must not decrease");
  if (k > 0) {
    b = &s->bufs[bi];  // the buffer the pass copied into
    if (frames->schema_allow) open_rule(b);
    if (b->has_rule)
      write_rule(b, b->questions, qs, frames->schema_allow, frames->schema_allow ? frames->band_allow : nullptr);
    uint64_t rr = b->records;
    for (uint32_t f = 0; f < k; f++) {
      rr += ro[f + 1] - ro[f];
      b->rec_off[b->frames + f + 1] = rr;
    }
    b->records += recs;
    b->questions += qs;
    b->p_total += ps;
    b->frames += k;
    if (first_ticket) *first_ticket = s->next_ticket;
    s->next_ticket += k;
    if (pushed) *pushed = k;
  }
  const ThreadUsage u1 = thread_usage();
  int cpu, node;
  where_am_i(&cpu, &node);
  kc_stream_stats& x = s->stats;
  x.push_calls++;
  x.frames_pushed += k;
  x.bytes_staged += recs * 72 + (k && s->bufs[bi].has_rule ? qs * 36 : 0);
  x.push_ms += steady_ms() - t0;
  x.caller_minor_faults += u1.minflt - u0.minflt;
  x.caller_involuntary_switches += u1.nivcsw - u0.nivcsw;
  x.caller_numa_node = node;
  return st;
}

kc_status kc_stream_flush(kc_stream* s) {
  if (!s) return KC_ERR_INVALID_ARG;
  {
    std::lock_guard<std::mutex> pl(s->push_mu);
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
  out->started_ms = b.start_ms;
  out->sync_wait_ms = b.wait_ms;
  return KC_OK;
}

kc_status kc_stream_read_stats(kc_stream* s, int reset, kc_stream_stats* out) {
  if (!s || !out) return KC_ERR_INVALID_ARG;
  std::lock_guard<std::mutex> pl(s->push_mu);
  std::lock_guard<std::mutex> lk(s->mu);
  *out = s->stats;
  if (reset) {
    kc_stream_stats keep{};
    keep.gpu_numa_node = s->stats.gpu_numa_node;
    keep.staging_numa_node = s->stats.staging_numa_node;
    keep.worker_numa_node = s->stats.worker_numa_node;
    keep.caller_numa_node = s->stats.caller_numa_node;
    keep.push_threads = s->stats.push_threads;
    keep.bound_cpus = s->stats.bound_cpus;
    s->stats = keep;
  }
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
  s->pool.shut();
  for (StreamBuf& b : s->bufs) free_buf(b);
  delete s;
}

}  // extern "C"
