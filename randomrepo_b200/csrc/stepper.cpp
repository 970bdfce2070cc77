// Native host path of one decode step (C ABI in include/pkv_b200.h).
//
// One call per step does what the Python layer would otherwise do in many:
// the allocator's per-token append for every sequence of the batch, the
// device upload and application of any pending block-table updates, the
// split-K plan, and one staged upload of the step descriptor; one call per
// layer then launches the fused decode kernels.  Host buffers are pinned and
// recycled through a small ring (one CUDA event per trip round the ring guards
// their reuse), device buffers are recycled in stream order, so a step costs
// a few CUDA calls of host time and never synchronises the host with the
// device.
//
// Everything a stepper launches goes to the stream passed to begin(); use one
// stream per stepper.

#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cstring>
#include <string>
#include <vector>

#include "pkv_b200.h"
#include "pkv_error.h"
#include "pkv_internal.h"

namespace {

constexpr int kRing = 8;

struct Slot {
  int32_t* host = nullptr;
  int32_t* dev = nullptr;
  int64_t cap = 0;  // int32 elements
};

int32_t cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return PKV_OK;
  pkv_set_error(std::string(what) + ": " + cudaGetErrorString(e));
  return PKV_ERR_CUDA;
}

}  // namespace

struct pkv_stepper {
  pkv_allocator* alloc = nullptr;
  pkv_pool_geom geom{};
  void* pool = nullptr;
  int num_sms = 148;
  int32_t* tables = nullptr;
  int32_t stride = 0;
  int32_t rows = 0;
  int32_t* lens = nullptr;
  int32_t* refs = nullptr;
  Slot slot[kRing];
  int next = 0;
  int last_taken = -1;
  // Recorded after the copy out of the ring's last slot; every copy of that
  // trip round the ring is complete once it is, so it guards the reuse of
  // all kRing slots (one event per kRing uploads instead of one per upload).
  cudaEvent_t round_done = nullptr;
  bool round_pending = false;
  // Descriptor uploads on their own stream: the copy for step i+1 runs while
  // step i's kernels do; the step's kernels wait for it through copy_ev, and
  // the first copy of each trip round the ring waits (on the device) for the
  // kernels enqueued before it, which read the slots it is about to reuse.
  cudaStream_t copy_stream = nullptr;
  cudaEvent_t copy_ev = nullptr, reuse_ev = nullptr;
  // Host-buffer steps (pkv_stepper_step_host): device staging of q / k / v
  // and of the output in kIo entries used in turn, in rounds of kIoRound.  A
  // step's inputs cross on copy_stream ahead of its descriptor (so the one
  // wait on copy_ev covers both), its output crosses on d2h_stream after its
  // kernels (k_done).  Reuse is guarded once per round, a round behind: the
  // first step of round r records the kernels and output copies enqueued so
  // far (in_ev / out_ev [r % 2]) and waits for those recorded at the start
  // of round r - 1, i.e. for round r - 2, the last one that used these
  // entries -- long finished, so the guard never stalls the pipeline.  A step
  // costs three CUDA calls beyond a device-buffer step.
  static constexpr int kIoRound = kRing;
  static constexpr int kIo = 2 * kIoRound;
  struct Io {
    char* in = nullptr;
    char* out = nullptr;
    int64_t in_cap = 0, out_cap = 0;
  };
  Io io[kIo];
  int io_next = 0;
  int io_cur = -1;        // entry of the step whose inputs were staged last
  int64_t io_in_round = 0;   // rounds begun on the staging side
  int64_t io_cur_round = 0;  // round of the entry staged last
  int64_t out_ev_round[2] = {-1, -1};  // round whose start each out_ev records
  bool io_out_issued = false;
  int64_t io_q_bytes = 0, io_kv_bytes = 0;
  int32_t io_batch = 0;
  cudaStream_t d2h_stream = nullptr;
  cudaEvent_t in_ev[2] = {}, out_ev[2] = {}, k_done = nullptr, fence_ev = nullptr;
  bool round_open = false;  // the ring's last slot was taken and not yet copied out
  std::vector<int32_t> rows_h, lens_h, newb_h, tokb_h, plan_h, upd_h;
  std::vector<int32_t> last_copies;  // (src, dst) pairs applied by the last sync / upload
  // Optional host array of per-block stored-token counts (the store's
  // bookkeeping of which blocks hold data): copy-on-write copies carry the
  // source's count, and each step sets the count of the block its token went to.
  int32_t* fill = nullptr;
  int64_t fill_n = 0;
  pkv_step_info info{};
  bool step_ready = false;
  void* ws = nullptr;
  int64_t ws_bytes = 0;
  cudaStream_t ws_stream = nullptr;
  int64_t launches = 0;
  // Length / refcount updates uploaded with the step descriptor, applied by
  // the step's first decode launch (device pointer past the drain header).
  const int32_t* def_dev = nullptr;
  int32_t def_refs = 0, def_lens = 0;
  bool def_pending = false;
  // Fixed-step mode: every step's descriptor goes to the same device block,
  // whose header gives the kernels the step's counts, so the attention
  // launches of a step can be recorded once in a CUDA graph and replayed.
  // Layout (int32): header[16] | deferred updates | slots (int64) | rows |
  // lens | new blocks | combine entries (int4) | work items (int4).
  bool fixed = false;
  int32_t fx_batch = 0, fx_items = 0, fx_combine = 0;
  int64_t fx_def_cap = 0, fx_off_def = 0, fx_off_slots = 0, fx_off_rows = 0, fx_off_comb = 0, fx_off_items = 0;
  int32_t* fx_dev = nullptr;
  std::vector<int32_t> fx_plan;
  // Optional per-launch timing of the decode kernels (events around them).
  std::vector<cudaEvent_t> t_start, t_stop;
  int64_t t_cap = 0, t_count = 0, t_every = 1, t_seen = 0;
  // Host time spent blocked on the staging ring (the host ran kRing steps
  // ahead of the device), so that callers can tell host work from waiting.
  int64_t wait_ns = 0;

  ~pkv_stepper() {
    if (round_done) {
      cudaEventSynchronize(round_done);
      cudaEventDestroy(round_done);
    }
    if (copy_stream) {
      cudaStreamSynchronize(copy_stream);
      cudaStreamDestroy(copy_stream);
      cudaEventDestroy(copy_ev);
      cudaEventDestroy(reuse_ev);
    }
    if (d2h_stream) {
      cudaStreamSynchronize(d2h_stream);
      cudaStreamDestroy(d2h_stream);
    }
    for (auto& e : io) {
      if (e.in) cudaFree(e.in);
      if (e.out) cudaFree(e.out);
    }
    for (auto ev : {in_ev[0], in_ev[1], out_ev[0], out_ev[1], k_done, fence_ev})
      if (ev) cudaEventDestroy(ev);
    for (auto& s : slot) {
      if (s.host) cudaFreeHost(s.host);
      if (s.dev) cudaFree(s.dev);
    }
    if (ws) cudaFree(ws);
    if (fx_dev) cudaFree(fx_dev);
    for (auto e : t_start) cudaEventDestroy(e);
    for (auto e : t_stop) cudaEventDestroy(e);
  }

  // A ring slot with room for `n` int32, its previous upload finished.
  int32_t take_slot(int64_t n, Slot** out) {
    if (next == 0 && round_pending) {
      const auto t0 = std::chrono::steady_clock::now();
      int32_t st = cuda_status(cudaEventSynchronize(round_done), "stepper ring");
      wait_ns += std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - t0).count();
      if (st) return st;
      round_pending = false;
    } else if (next == 0 && round_open) {
      // A failed call took the last slot without copying it out, so no event
      // closes that round: wait for the device instead (error paths only).
      int32_t st = cuda_status(cudaDeviceSynchronize(), "stepper ring");
      if (st) return st;
    }
    round_open = next == kRing - 1;
    Slot& s = slot[next];
    last_taken = next;
    next = (next + 1) % kRing;
    if (s.cap < n) {
      // Grow this slot and every later one of the round together (none of
      // them is in flight: the round began after the previous one's copies
      // ended), so that a run of steps allocates once, not once per slot.
      const int64_t cap = std::max<int64_t>({n + n / 4, 2 * s.cap, 4096});
      for (int j = last_taken; j < kRing; ++j) {
        Slot& x = slot[j];
        if (x.cap >= cap) continue;
        if (x.host) cudaFreeHost(x.host);
        if (x.dev) cudaFree(x.dev);  // implicit device sync: only when slots grow
        x.host = nullptr;
        x.dev = nullptr;
        x.cap = 0;
        int32_t st = cuda_status(cudaHostAlloc((void**)&x.host, cap * 4, cudaHostAllocDefault), "cudaHostAlloc");
        if (!st) st = cuda_status(cudaMalloc((void**)&x.dev, cap * 4), "cudaMalloc");
        if (st) return st;
        x.cap = cap;
      }
    }
    *out = &s;
    return PKV_OK;
  }

  // After the copy out of the slot last taken: close the trip round the ring.
  int32_t copied(cudaStream_t stream) {
    if (last_taken != kRing - 1) return PKV_OK;
    round_open = false;
    if (!round_done) {
      int32_t st = cuda_status(cudaEventCreateWithFlags(&round_done, cudaEventDisableTiming), "cudaEventCreate");
      if (st) return st;
    }
    int32_t st = cuda_status(cudaEventRecord(round_done, stream), "cudaEventRecord");
    if (!st) round_pending = true;
    return st;
  }

  // The step descriptor into the fixed block (fixed-step mode).
  int32_t upload_fixed(cudaStream_t cs, pkv_step_info* out_info, int32_t n, int32_t pps, int64_t n_items,
                       int64_t n_combine, bool defer, int64_t pr, int64_t pl) {
    if (n > fx_batch || n_items > fx_items || n_combine > fx_combine) {
      pkv_set_error("decode step exceeds the fixed-step capacity (" + std::to_string(n) + " sequences, " +
                    std::to_string(n_items) + " work items; capacity " + std::to_string(fx_batch) + ", " +
                    std::to_string(fx_items) + ")");
      if (n <= fx_batch) out_info->need_items = (int32_t)n_items;
      return PKV_ERR_UNSUPPORTED;
    }
    if (defer && 4 + 2 * (pr + pl) > fx_def_cap) {
      // Too many pending updates for the block: apply them with the table kernel.
      int32_t n_copies = 0;
      int32_t s = apply_pending(cs, nullptr, 0, &n_copies);
      if (s) return s;
      defer = false;
    }
    const int64_t used = fx_off_items + 4 * n_items;
    Slot* sl;
    int32_t s = take_slot(fx_off_items + 4 * (int64_t)fx_items, &sl);
    if (s) return s;
    int32_t* h = sl->host;
    fx_plan.resize(4 * (n_items + n_combine));
    s = pkv_decode_plan(lens_h.data(), n, geom.num_kv_heads, geom.head_dim, num_sms, &pps, fx_plan.data(),
                        n_items + n_combine, &n_items, &n_combine);
    if (s) return s;
    std::memcpy(h + fx_off_items, fx_plan.data(), 4 * n_items * 4);
    std::memcpy(h + fx_off_comb, fx_plan.data() + 4 * n_items, 4 * n_combine * 4);
    int64_t written = 0;
    if (defer) {
      s = pkv_allocator_drain_updates(alloc, h + fx_off_def, fx_def_cap, &written);
      if (s) return s;
    }
    std::memset(h, 0, 16 * 4);
    h[0] = (int32_t)n_items;
    h[1] = (int32_t)n_combine;
    h[2] = n;
    h[3] = pps;
    h[4] = defer ? h[fx_off_def + 1] : 0;
    h[5] = defer ? h[fx_off_def + 2] : 0;
    int64_t* slots = reinterpret_cast<int64_t*>(h + fx_off_slots);
    const int32_t bs = geom.block_size;
    for (int i = 0; i < n; ++i) slots[i] = (int64_t)tokb_h[i] * bs + (lens_h[i] - 1) % bs;
    std::memcpy(h + fx_off_rows, rows_h.data(), n * 4);
    std::memcpy(h + fx_off_rows + fx_batch, lens_h.data(), n * 4);
    std::memcpy(h + fx_off_rows + 2 * fx_batch, newb_h.data(), n * 4);
    s = cuda_status(cudaMemcpyAsync(fx_dev, h, used * 4, cudaMemcpyHostToDevice, cs), "H2D");
    if (!s) s = copied(cs);
    if (s) return s;
    if (fill) {
      for (int i = 0; i < n; ++i) {
        const int32_t b = tokb_h[i];
        if (b >= 0 && b < fill_n) fill[b] = (lens_h[i] - 1) % bs + 1;
      }
    }
    def_pending = false;
    out_info->pages_per_split = pps;
    out_info->n_items = (int32_t)n_items;
    out_info->n_combine = (int32_t)n_combine;
    out_info->items = fx_dev + fx_off_items;
    out_info->slots = reinterpret_cast<const int64_t*>(fx_dev + fx_off_slots);
    out_info->rows = fx_dev + fx_off_rows;
    out_info->seq_lens = fx_dev + fx_off_rows + fx_batch;
    out_info->new_blocks = fx_dev + fx_off_rows + 2 * fx_batch;
    info = *out_info;
    step_ready = true;
    return PKV_OK;
  }

  int32_t ensure_copy_stream() {
    if (copy_stream) return PKV_OK;
    int32_t st = cuda_status(cudaStreamCreateWithFlags(&copy_stream, cudaStreamNonBlocking), "cudaStreamCreate");
    if (!st) st = cuda_status(cudaEventCreateWithFlags(&copy_ev, cudaEventDisableTiming), "cudaEventCreate");
    if (!st) st = cuda_status(cudaEventCreateWithFlags(&reuse_ev, cudaEventDisableTiming), "cudaEventCreate");
    return st;
  }

  int32_t upload(Slot* s, int64_t n, cudaStream_t stream) {
    if (int32_t e = ensure_copy_stream()) return e;
    if (last_taken == 0) {
      int32_t st = cuda_status(cudaEventRecord(reuse_ev, stream), "cudaEventRecord");
      if (!st) st = cuda_status(cudaStreamWaitEvent(copy_stream, reuse_ev, 0), "cudaStreamWaitEvent");
      if (st) return st;
    }
    int32_t st = cuda_status(cudaMemcpyAsync(s->dev, s->host, n * 4, cudaMemcpyHostToDevice, copy_stream), "H2D");
    if (!st) st = cuda_status(cudaEventRecord(copy_ev, copy_stream), "cudaEventRecord");
    if (!st) st = cuda_status(cudaStreamWaitEvent(stream, copy_ev, 0), "cudaStreamWaitEvent");
    return st ? st : copied(copy_stream);
  }

  // The output stream and the staging guards' events (on first use).
  int32_t ensure_host_io() {
    if (d2h_stream) return PKV_OK;
    int32_t st = cuda_status(cudaStreamCreateWithFlags(&d2h_stream, cudaStreamNonBlocking), "cudaStreamCreate");
    for (cudaEvent_t* ev : {&in_ev[0], &in_ev[1], &out_ev[0], &out_ev[1], &k_done, &fence_ev})
      if (!st) st = cuda_status(cudaEventCreateWithFlags(ev, cudaEventDisableTiming), "cudaEventCreate");
    return st;
  }

  // Copy a step's host q / k / v into the next staging entry on copy_stream
  // (one copy when the caller says the three are consecutive parts of one
  // allocation: adjacent addresses alone do not make one copyable range).
  int32_t stage_inputs(int32_t n, int32_t num_q_heads, const void* q, const void* k, const void* v, bool packed,
                       cudaStream_t stream) {
    if (int32_t e = ensure_copy_stream()) return e;
    if (int32_t e = ensure_host_io()) return e;
    const int64_t eb = geom.dtype == PKV_F32 ? 4 : 2;
    const int64_t qb = (int64_t)n * num_q_heads * geom.head_dim * eb;
    const int64_t kb = k ? (int64_t)n * geom.num_kv_heads * geom.head_dim * eb : 0;
    const int64_t in_need = qb + 2 * kb;
    Io& e = io[io_next];
    if (e.in_cap < in_need || e.out_cap < qb) {
      // Grow (rare) every entry at once, so that the steps that follow
      // allocate nothing: after the device has finished with the old buffers.
      bool any = false;
      for (const Io& x : io) any = any || x.in || x.out;
      if (any) {
        if (int32_t st = cuda_status(cudaDeviceSynchronize(), "host-step staging")) return st;
      }
      const int64_t in_cap = std::max<int64_t>(in_need, 1 << 20), out_cap = std::max<int64_t>(qb, 1 << 20);
      for (Io& x : io) {
        if (x.in) cudaFree(x.in);
        if (x.out) cudaFree(x.out);
        x.in = x.out = nullptr;
        x.in_cap = x.out_cap = 0;
      }
      for (Io& x : io) {
        int32_t st = cuda_status(cudaMalloc((void**)&x.in, in_cap), "cudaMalloc host-step staging");
        if (!st) st = cuda_status(cudaMalloc((void**)&x.out, out_cap), "cudaMalloc host-step staging");
        if (st) return st;
        x.in_cap = in_cap;
        x.out_cap = out_cap;
      }
    }
    // First entry of a round r: record the kernels enqueued so far (through
    // round r - 1) and let this round's copies wait for round r - 2's.
    if (io_next % kIoRound == 0) {
      const int64_t r = io_in_round++;
      int32_t st = PKV_OK;
      if (r >= 1) st = cuda_status(cudaEventRecord(in_ev[r % 2], stream), "cudaEventRecord");
      if (!st && r >= 2) st = cuda_status(cudaStreamWaitEvent(copy_stream, in_ev[(r - 1) % 2], 0), "cudaStreamWaitEvent");
      if (st) return st;
    }
    const char* qc = static_cast<const char*>(q);
    int32_t st;
    if (!k || (packed && static_cast<const char*>(k) == qc + qb && static_cast<const char*>(v) == qc + qb + kb)) {
      st = cuda_status(cudaMemcpyAsync(e.in, q, in_need, cudaMemcpyHostToDevice, copy_stream), "H2D q/k/v");
    } else {
      st = cuda_status(cudaMemcpyAsync(e.in, q, qb, cudaMemcpyHostToDevice, copy_stream), "H2D q");
      if (!st) st = cuda_status(cudaMemcpyAsync(e.in + qb, k, kb, cudaMemcpyHostToDevice, copy_stream), "H2D k");
      if (!st) st = cuda_status(cudaMemcpyAsync(e.in + qb + kb, v, kb, cudaMemcpyHostToDevice, copy_stream), "H2D v");
    }
    if (st) return st;
    io_cur = io_next;
    io_cur_round = io_in_round - 1;
    io_next = (io_next + 1) % kIo;
    io_q_bytes = qb;
    io_kv_bytes = kb;
    io_batch = n;
    return PKV_OK;
  }

  bool capacity_ok(pkv_step_info* out) {
    pkv_allocator_stats stats;
    pkv_allocator_get_stats(alloc, &stats);
    out->need_rows = (int32_t)stats.row_capacity;
    out->need_cols = (int32_t)stats.max_blocks_per_row;
    return tables && stats.row_capacity <= rows && stats.max_blocks_per_row <= stride;
  }

  // Deferred updates that no decode launch consumed go through the table
  // kernel before anything else reads the mirror.
  int32_t flush_deferred(cudaStream_t stream) {
    if (!def_pending) return PKV_OK;
    def_pending = false;
    const int32_t header[4] = {0, def_refs, def_lens, 0};
    launches += 1;
    return pkv_apply_updates(&geom, pool, tables, stride, rows, refs, lens, def_dev - 4, header, stream);
  }

  // Drain the allocator's pending table / refcount / length updates and
  // copy-on-write copies, and apply them on `stream`.
  int32_t apply_pending(cudaStream_t stream, int32_t* copies_out, int64_t copies_cap, int32_t* n_copies) {
    int32_t fs = flush_deferred(stream);
    if (fs) return fs;
    int64_t nt, nr, nl, nc;
    pkv_allocator_pending_updates(alloc, &nt, &nr, &nl, &nc);
    *n_copies = 0;
    if (nt + nr + nl + nc == 0) return PKV_OK;
    const int64_t cap = 4 + 3 * nt + 2 * nr + 2 * nl + 2 * nc;
    Slot* s;
    int32_t st = take_slot(cap, &s);
    if (st) return st;
    int64_t written = 0;
    st = pkv_allocator_drain_updates(alloc, s->host, cap, &written);
    if (st) return st;
    last_copies.clear();
    if (s->host[3] > 0) {
      const int64_t off = 4 + 3 * (int64_t)s->host[0] + 2 * (int64_t)s->host[1] + 2 * (int64_t)s->host[2];
      last_copies.assign(s->host + off, s->host + off + 2 * (int64_t)s->host[3]);
      if (copies_out) {
        const int64_t n = std::min<int64_t>(s->host[3], copies_cap);
        std::memcpy(copies_out, s->host + off, n * 2 * 4);
      }
    }
    *n_copies = s->host[3];
    if (fill) {
      for (size_t i = 0; i + 1 < last_copies.size(); i += 2) {
        const int32_t src = last_copies[i], dst = last_copies[i + 1];
        if (src >= 0 && src < fill_n && dst >= 0 && dst < fill_n) fill[dst] = fill[src];
      }
    }
    st = cuda_status(cudaMemcpyAsync(s->dev, s->host, written * 4, cudaMemcpyHostToDevice, stream), "H2D");
    if (st) return st;
    st = pkv_apply_updates(&geom, pool, tables, stride, rows, refs, lens, s->dev, s->host, stream);
    // The host copy is read by pkv_apply_updates synchronously; the ring's
    // event only guards the pinned buffer against reuse before the H2D completes.
    int32_t st2 = copied(stream);
    launches += 1 + (s->host[3] > 0 ? 1 : 0);
    return st ? st : st2;
  }
};

extern "C" {

pkv_stepper* pkv_stepper_create(pkv_allocator* a, const pkv_pool_geom* g, void* pool, int32_t* status) {
  pkv_clear_error();
  if (!a || !g || !pool) {
    pkv_set_error("pkv_stepper_create: null argument");
    if (status) *status = PKV_ERR_ARG;
    return nullptr;
  }
  auto* st = new pkv_stepper();
  st->alloc = a;
  st->geom = *g;
  st->pool = pool;
  int dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&st->num_sms, cudaDevAttrMultiProcessorCount, dev);
  if (st->num_sms <= 0) st->num_sms = 148;
  if (status) *status = PKV_OK;
  return st;
}

void pkv_stepper_destroy(pkv_stepper* st) { delete st; }

int32_t pkv_stepper_bind_tables(pkv_stepper* st, int32_t* block_tables, int32_t table_stride, int32_t table_rows,
                                int32_t* context_lens, int32_t* refcounts) {
  st->tables = block_tables;
  st->stride = table_stride;
  st->rows = table_rows;
  st->lens = context_lens;
  st->refs = refcounts;
  return PKV_OK;
}

int32_t pkv_stepper_fix_steps(pkv_stepper* st, int32_t max_batch, int32_t max_items, void* stream) {
  pkv_clear_error();
  if (max_batch <= 0 || max_items < 0) {
    pkv_set_error("pkv_stepper_fix_steps: max_batch must be positive and max_items non-negative");
    return PKV_ERR_ARG;
  }
  const int32_t hpc = pkv_decode_heads_per_item(st->geom.num_kv_heads);
  const int32_t groups = st->geom.num_kv_heads / hpc;
  const int32_t warps = st->num_sms * (2 * 16 * st->geom.head_dim * 2 * hpc >= 16384 ? PKV_DECODE_WARPS_BIG : 8);
  if (max_items == 0) max_items = groups * max_batch + 4 * warps;
  max_items = std::max(max_items, groups * max_batch);
  auto cs = static_cast<cudaStream_t>(stream);
  if (st->fx_dev) {
    int32_t s0 = cuda_status(cudaStreamSynchronize(cs), "pkv_stepper_fix_steps");
    if (s0) return s0;
    cudaFree(st->fx_dev);
    st->fx_dev = nullptr;
  }
  st->fixed = false;
  st->fx_batch = max_batch;
  st->fx_items = max_items;
  st->fx_combine = groups * max_batch;
  st->fx_def_cap = 4 + 4 * (int64_t)max_batch + 256;
  st->fx_off_def = 16;
  st->fx_off_slots = st->fx_off_def + st->fx_def_cap;        // even: int64-aligned
  st->fx_off_rows = st->fx_off_slots + 2 * (int64_t)max_batch;
  st->fx_off_comb = (st->fx_off_rows + 3 * (int64_t)max_batch + 3) & ~int64_t(3);  // int4-aligned
  st->fx_off_items = st->fx_off_comb + 4 * (int64_t)st->fx_combine;
  const int64_t total = st->fx_off_items + 4 * (int64_t)max_items;
  int32_t s = cuda_status(cudaMalloc((void**)&st->fx_dev, total * 4), "cudaMalloc fixed step block");
  if (!s) s = cuda_status(cudaMemsetAsync(st->fx_dev, 0, total * 4, cs), "cudaMemsetAsync fixed step block");
  if (s) return s;
  // The workspace for the capacities, allocated now so that no step allocates.
  const int64_t need = pkv_decode_workspace_bytes(max_batch, st->geom.num_kv_heads, st->geom.head_dim, max_items);
  if (need > st->ws_bytes) {
    if (st->ws) {
      s = cuda_status(cudaStreamSynchronize(cs), "stepper workspace");
      if (s) return s;
      cudaFree(st->ws);
      st->ws = nullptr;
    }
    s = cuda_status(cudaMalloc(&st->ws, need), "cudaMalloc workspace");
    if (!s) s = cuda_status(cudaMemsetAsync(st->ws, 0, need, cs), "cudaMemsetAsync workspace");
    if (s) return s;
    st->ws_bytes = need;
  }
  st->fixed = true;
  st->step_ready = false;
  return PKV_OK;
}

int32_t pkv_stepper_fixed_capacity(pkv_stepper* st, int32_t* max_batch, int32_t* max_items) {
  *max_batch = st->fixed ? st->fx_batch : 0;
  *max_items = st->fixed ? st->fx_items : 0;
  return PKV_OK;
}

int32_t pkv_stepper_bind_fill(pkv_stepper* st, int32_t* block_fill, int64_t n_blocks) {
  pkv_clear_error();
  if (n_blocks < 0 || (n_blocks > 0 && !block_fill)) {
    pkv_set_error("pkv_stepper_bind_fill: invalid arguments");
    return PKV_ERR_ARG;
  }
  st->fill = n_blocks ? block_fill : nullptr;
  st->fill_n = n_blocks;
  return PKV_OK;
}

int32_t pkv_stepper_sync(pkv_stepper* st, void* stream, int32_t* copies_out, int64_t copies_cap, int32_t* n_copies,
                         int32_t* need_rows, int32_t* need_cols) {
  pkv_clear_error();
  pkv_step_info probe{};
  if (!st->capacity_ok(&probe)) {
    *need_rows = probe.need_rows;
    *need_cols = probe.need_cols;
    pkv_set_error("device block tables too small");
    return PKV_ERR_CAPACITY;
  }
  return st->apply_pending(static_cast<cudaStream_t>(stream), copies_out, copies_cap, n_copies);
}

int32_t pkv_stepper_begin(pkv_stepper* st, const int64_t* sequence_ids, int32_t n, pkv_step_info* info,
                          int32_t* rows_out, int32_t* lens_out, int32_t* token_blocks_out) {
  pkv_clear_error();
  st->step_ready = false;
  if (n <= 0 || !sequence_ids || !info) {
    pkv_set_error("pkv_stepper_begin: invalid arguments");
    return PKV_ERR_ARG;
  }
  st->rows_h.resize(n);
  st->lens_h.resize(n);
  st->newb_h.resize(n);
  st->tokb_h.resize(n);
  int64_t done = 0;
  int32_t s = pkv_allocator_decode_step(st->alloc, sequence_ids, n, st->rows_h.data(), st->lens_h.data(),
                                        st->newb_h.data(), st->tokb_h.data(), &done);
  std::memset(info, 0, sizeof(*info));
  info->batch = (int32_t)done;
  if (rows_out) std::memcpy(rows_out, st->rows_h.data(), done * 4);
  if (lens_out) std::memcpy(lens_out, st->lens_h.data(), done * 4);
  if (token_blocks_out) std::memcpy(token_blocks_out, st->tokb_h.data(), done * 4);
  if (s != PKV_OK) {
    // The appends already made stay (as with the reference's sequential
    // append_tokens calls); record their rows so the next sync uploads them.
    pkv_allocator_touch_rows(st->alloc, st->rows_h.data(), done);
    st->rows_h.clear();
    return s;
  }
  return PKV_OK;
}

int32_t pkv_stepper_upload(pkv_stepper* st, void* stream, pkv_step_info* info, int32_t* copies_out,
                           int64_t copies_cap) {
  pkv_clear_error();
  auto cs = static_cast<cudaStream_t>(stream);
  const int32_t n = info->batch;
  if (n <= 0 || (size_t)n != st->rows_h.size()) {
    pkv_set_error("pkv_stepper_upload: no step begun");
    return PKV_ERR_ARG;
  }
  if (!st->capacity_ok(info)) {
    pkv_set_error("device block tables too small");
    return PKV_ERR_CAPACITY;
  }
  int32_t n_copies = 0;
  int32_t s = st->flush_deferred(cs);
  if (s) return s;
  int64_t pt, pr, pl, pc;
  pkv_allocator_pending_updates(st->alloc, &pt, &pr, &pl, &pc);
  // Only lengths / refcounts pending (the decode never reads them): they ride
  // in the descriptor upload and the decode kernel applies them.
  const bool defer = pt == 0 && pc == 0 && pr + pl > 0;
  st->last_copies.clear();
  if (!defer) {
    s = st->apply_pending(cs, copies_out, copies_cap, &n_copies);
    if (s) return s;
  }
  info->n_copies = n_copies;
  int32_t pps = 0;
  int64_t n_items = 0, n_combine = 0;
  s = pkv_decode_plan(st->lens_h.data(), n, st->geom.num_kv_heads, st->geom.head_dim, st->num_sms, &pps, nullptr, 0,
                      &n_items, &n_combine);
  if (s) return s;
  if (st->fixed) return st->upload_fixed(cs, info, n, pps, n_items, n_combine, defer, pr, pl);
  // Descriptor: [items + combine entries (int4) | slots (int64) | rows | lens | new_blocks]
  const int64_t n_quads = n_items + n_combine;
  const int64_t def_off = 4 * n_quads + 2 * n + 3 * n;
  const int64_t def_cap = defer ? 4 + 2 * (pr + pl) : 0;
  const int64_t total = def_off + def_cap;
  Slot* sl;
  s = st->take_slot(total, &sl);
  if (s) return s;
  int32_t* h = sl->host;
  s = pkv_decode_plan(st->lens_h.data(), n, st->geom.num_kv_heads, st->geom.head_dim, st->num_sms, &pps, h, n_quads,
                      &n_items, &n_combine);
  if (s) return s;
  int64_t* slots = reinterpret_cast<int64_t*>(h + 4 * n_quads);
  const int32_t bs = st->geom.block_size;
  for (int i = 0; i < n; ++i) slots[i] = (int64_t)st->tokb_h[i] * bs + (st->lens_h[i] - 1) % bs;
  int32_t* tail = h + 4 * n_quads + 2 * n;
  std::memcpy(tail, st->rows_h.data(), n * 4);
  std::memcpy(tail + n, st->lens_h.data(), n * 4);
  std::memcpy(tail + 2 * n, st->newb_h.data(), n * 4);
  int64_t written = 0;
  if (defer) {
    s = pkv_allocator_drain_updates(st->alloc, h + def_off, def_cap, &written);
    if (s) return s;
  }
  s = st->upload(sl, def_off + written, cs);
  if (s) return s;
  int32_t* d = sl->dev;
  if (defer) {
    st->def_dev = d + def_off + 4;
    st->def_refs = h[def_off + 1];
    st->def_lens = h[def_off + 2];
    st->def_pending = true;
  }
  if (st->fill) {
    // After any copy-on-write copies (they carry the source block's count).
    for (int i = 0; i < n; ++i) {
      const int32_t b = st->tokb_h[i];
      if (b >= 0 && b < st->fill_n) st->fill[b] = (st->lens_h[i] - 1) % bs + 1;
    }
  }
  info->pages_per_split = pps;
  info->n_items = (int32_t)n_items;
  info->n_combine = (int32_t)n_combine;
  info->items = d;
  info->slots = reinterpret_cast<const int64_t*>(d + 4 * n_quads);
  info->rows = d + 4 * n_quads + 2 * n;
  info->seq_lens = info->rows + n;
  info->new_blocks = info->rows + 2 * n;
  // Workspace for this plan (grown rarely; a new one starts zeroed).
  const int64_t need = pkv_decode_workspace_bytes(n, st->geom.num_kv_heads, st->geom.head_dim, n_items);
  if (need > st->ws_bytes) {
    if (st->ws) {
      s = cuda_status(cudaStreamSynchronize(cs), "stepper workspace");
      if (s) return s;
      cudaFree(st->ws);
      st->ws = nullptr;
    }
    const int64_t bytes = std::max<int64_t>(need, (int64_t)1 << 20) * 2;
    s = cuda_status(cudaMalloc(&st->ws, bytes), "cudaMalloc workspace");
    if (!s) s = cuda_status(cudaMemsetAsync(st->ws, 0, bytes, cs), "cudaMemsetAsync workspace");
    if (s) return s;
    st->ws_bytes = bytes;
  }
  st->info = *info;
  st->step_ready = true;
  return PKV_OK;
}

int32_t pkv_stepper_attention(pkv_stepper* st, int32_t layer, const void* q, const void* k_new, const void* v_new,
                              int32_t num_q_heads, float scale, void* out, void* stream) {
  if (!st->step_ready) {
    pkv_clear_error();
    pkv_set_error("pkv_stepper_attention: no step uploaded");
    return PKV_ERR_ARG;
  }
  const pkv_step_info& in = st->info;
  const bool timed = st->t_count < st->t_cap && (st->t_seen++ % st->t_every) == 0;
  if (st->fixed) {
    // Same arguments every step: capacities, the fixed block, its header.
    if (timed) cudaEventRecord(st->t_start[st->t_count], static_cast<cudaStream_t>(stream));
    int32_t s = pkv_decode_attention_ex(&st->geom, st->pool, layer, q, k_new, v_new, st->tables, st->stride,
                                        st->rows, st->lens, in.rows, in.seq_lens, in.new_blocks, in.items,
                                        st->fx_items, st->fx_combine, st->fx_batch, num_q_heads, 1, scale, out,
                                        st->ws, st->ws_bytes, stream, st->fx_dev + st->fx_off_def + 4, 0, 0,
                                        st->refs, st->fx_dev, st->fx_dev + st->fx_off_comb);
    if (timed) cudaEventRecord(st->t_stop[st->t_count++], static_cast<cudaStream_t>(stream));
    if (s == PKV_OK) st->launches += 2;
    return s;
  }
  const int32_t* def = st->def_pending ? st->def_dev : nullptr;
  if (timed) cudaEventRecord(st->t_start[st->t_count], static_cast<cudaStream_t>(stream));
  int32_t s = pkv_decode_attention_ex(&st->geom, st->pool, layer, q, k_new, v_new, st->tables, st->stride, st->rows,
                                      st->lens, in.rows, in.seq_lens, in.new_blocks, in.items, in.n_items,
                                      in.n_combine, in.batch, num_q_heads, in.pages_per_split, scale, out, st->ws,
                                      st->ws_bytes, stream, def, st->def_refs, st->def_lens, st->refs, nullptr,
                                      nullptr);
  if (s == PKV_OK && def) st->def_pending = false;
  if (timed) cudaEventRecord(st->t_stop[st->t_count++], static_cast<cudaStream_t>(stream));
  if (s == PKV_OK) st->launches += 1 + (in.n_combine > 0 ? 1 : 0);
  return s;
}

int32_t pkv_stepper_step(pkv_stepper* st, const int64_t* sequence_ids, int32_t n, int32_t layer, const void* q,
                         const void* k_new, const void* v_new, int32_t num_q_heads, float scale, void* out,
                         void* stream, pkv_step_info* info, int32_t* rows_out, int32_t* lens_out,
                         int32_t* token_blocks_out, int32_t* copies_out, int64_t copies_cap) {
  int32_t s = pkv_stepper_begin(st, sequence_ids, n, info, rows_out, lens_out, token_blocks_out);
  if (s) return s;
  s = pkv_stepper_upload(st, stream, info, copies_out, copies_cap);
  if (s) return s;  // PKV_ERR_CAPACITY: grow, rebind, then upload + attention
  return pkv_stepper_attention(st, layer, q, k_new, v_new, num_q_heads, scale, out, stream);
}

int32_t pkv_stepper_attention_host(pkv_stepper* st, int32_t layer, int32_t num_q_heads, float scale, void* out_host,
                                   void* stream) {
  if (st->io_cur < 0 || !st->step_ready || st->io_batch != st->info.batch) {
    pkv_clear_error();
    pkv_set_error("pkv_stepper_attention_host: no host step staged and uploaded");
    return PKV_ERR_ARG;
  }
  if (!out_host || num_q_heads <= 0 ||
      (int64_t)st->io_batch * num_q_heads * st->geom.head_dim * (st->geom.dtype == PKV_F32 ? 4 : 2) !=
          st->io_q_bytes) {
    pkv_clear_error();
    pkv_set_error("pkv_stepper_attention_host: output / head count does not match the staged step");
    return PKV_ERR_ARG;
  }
  auto cs = static_cast<cudaStream_t>(stream);
  const int ei = st->io_cur;
  auto& e = st->io[ei];
  st->io_cur = -1;
  // First entry of a round r: record the output copies enqueued so far
  // (through round r - 1) and let this round's kernels wait for round r - 2's
  // (recorded at the start of round r - 1; if that start was never reached --
  // a step abandoned after staging -- wait for every copy enqueued so far).
  if (ei % pkv_stepper::kIoRound == 0 && st->io_out_issued) {
    const int64_t r = st->io_cur_round;
    const int slot = (int)(r % 2), prev = 1 - slot;
    int32_t s = cuda_status(cudaEventRecord(st->out_ev[slot], st->d2h_stream), "cudaEventRecord");
    const bool have_prev = st->out_ev_round[prev] == r - 1;
    if (!s) s = cuda_status(cudaStreamWaitEvent(cs, have_prev ? st->out_ev[prev] : st->out_ev[slot], 0),
                            "cudaStreamWaitEvent");
    if (s) return s;
    st->out_ev_round[slot] = r;
  }
  const char* k = st->io_kv_bytes ? e.in + st->io_q_bytes : nullptr;
  const char* v = st->io_kv_bytes ? e.in + st->io_q_bytes + st->io_kv_bytes : nullptr;
  int32_t s = pkv_stepper_attention(st, layer, e.in, k, v, num_q_heads, scale, e.out, stream);
  if (s) return s;
  s = cuda_status(cudaEventRecord(st->k_done, cs), "cudaEventRecord");
  if (!s) s = cuda_status(cudaStreamWaitEvent(st->d2h_stream, st->k_done, 0), "cudaStreamWaitEvent");
  if (!s)
    s = cuda_status(cudaMemcpyAsync(out_host, e.out, st->io_q_bytes, cudaMemcpyDeviceToHost, st->d2h_stream),
                    "D2H out");
  if (s) return s;
  st->io_out_issued = true;
  return PKV_OK;
}

int32_t pkv_stepper_step_host(pkv_stepper* st, const int64_t* sequence_ids, int32_t n, int32_t layer,
                              const void* q_host, const void* k_new_host, const void* v_new_host,
                              int32_t inputs_packed, int32_t num_q_heads, float scale, void* out_host, void* stream, pkv_step_info* info,
                              int32_t* rows_out, int32_t* lens_out, int32_t* token_blocks_out) {
  if (!q_host || !out_host || num_q_heads <= 0 || num_q_heads % st->geom.num_kv_heads != 0 ||
      (!k_new_host) != (!v_new_host)) {
    pkv_clear_error();
    pkv_set_error("pkv_stepper_step_host: q and out are required, num_q_heads must be a positive multiple of the "
                  "KV heads, and k_new / v_new come together");
    return PKV_ERR_ARG;
  }
  int32_t s = pkv_stepper_begin(st, sequence_ids, n, info, rows_out, lens_out, token_blocks_out);
  if (s) return s;
  s = st->stage_inputs(n, num_q_heads, q_host, k_new_host, v_new_host, inputs_packed != 0,
                       static_cast<cudaStream_t>(stream));
  if (s) return s;
  s = pkv_stepper_upload(st, stream, info, nullptr, 0);
  if (s) return s;  // PKV_ERR_CAPACITY: grow, rebind, then upload + attention_host
  return pkv_stepper_attention_host(st, layer, num_q_heads, scale, out_host, stream);
}

int32_t pkv_host_alloc(int64_t bytes, int32_t write_combined, void** ptr_out) {
  pkv_clear_error();
  if (bytes <= 0 || !ptr_out) {
    pkv_set_error("pkv_host_alloc: bytes must be positive and ptr_out non-NULL");
    return PKV_ERR_ARG;
  }
  *ptr_out = nullptr;
  return cuda_status(cudaHostAlloc(ptr_out, (size_t)bytes,
                                   write_combined ? cudaHostAllocWriteCombined : cudaHostAllocDefault),
                     "cudaHostAlloc");
}

int32_t pkv_host_free(void* ptr) {
  pkv_clear_error();
  return ptr ? cuda_status(cudaFreeHost(ptr), "cudaFreeHost") : PKV_OK;
}

int32_t pkv_stepper_host_fence(pkv_stepper* st, void* stream) {
  pkv_clear_error();
  if (!st->io_out_issued) return PKV_OK;
  int32_t s = cuda_status(cudaEventRecord(st->fence_ev, st->d2h_stream), "cudaEventRecord");
  return s ? s : cuda_status(cudaStreamWaitEvent(static_cast<cudaStream_t>(stream), st->fence_ev, 0),
                             "cudaStreamWaitEvent");
}

int32_t pkv_stepper_copies(pkv_stepper* st, int32_t* pairs_out, int64_t capacity, int64_t* n_pairs) {
  const int64_t n = (int64_t)st->last_copies.size() / 2;
  *n_pairs = n;
  if (pairs_out) std::memcpy(pairs_out, st->last_copies.data(), std::min(n, capacity) * 2 * 4);
  return PKV_OK;
}

int32_t pkv_stepper_error(pkv_stepper* st, int32_t* device_error) {
  pkv_clear_error();
  *device_error = 0;
  if (!st->ws) return PKV_OK;
  return cuda_status(cudaMemcpy(device_error, st->ws, 4, cudaMemcpyDeviceToHost), "pkv_stepper_error");
}

int64_t pkv_stepper_launches(pkv_stepper* st) { return st->launches; }

int64_t pkv_stepper_host_wait_ns(pkv_stepper* st) { return st->wait_ns; }

int32_t pkv_stepper_time_launches(pkv_stepper* st, int64_t count, int64_t every) {
  pkv_clear_error();
  if (count < 0 || every < 1) {
    pkv_set_error("pkv_stepper_time_launches: count must be >= 0 and every >= 1");
    return PKV_ERR_ARG;
  }
  st->t_every = every;
  st->t_seen = 0;
  st->t_count = 0;
  if (count <= (int64_t)st->t_start.size()) {
    // The events made by an earlier call serve again: no CUDA call here, so
    // timing can be re-armed right before a timed region.
    st->t_cap = count;
    return PKV_OK;
  }
  for (auto e : st->t_start) cudaEventDestroy(e);
  for (auto e : st->t_stop) cudaEventDestroy(e);
  st->t_start.assign(count, nullptr);
  st->t_stop.assign(count, nullptr);
  for (int64_t i = 0; i < count; ++i) {
    int32_t s = cuda_status(cudaEventCreate(&st->t_start[i]), "cudaEventCreate");
    if (!s) s = cuda_status(cudaEventCreate(&st->t_stop[i]), "cudaEventCreate");
    if (s) {
      st->t_cap = 0;
      return s;
    }
  }
  st->t_cap = count;
  st->t_count = 0;
  return PKV_OK;
}

int32_t pkv_stepper_launch_times(pkv_stepper* st, float* ms_out, int64_t capacity, int64_t* n_out) {
  pkv_clear_error();
  const int64_t n = std::min(st->t_count, capacity);
  for (int64_t i = 0; i < n; ++i) {
    int32_t s = cuda_status(cudaEventSynchronize(st->t_stop[i]), "cudaEventSynchronize");
    if (!s) s = cuda_status(cudaEventElapsedTime(&ms_out[i], st->t_start[i], st->t_stop[i]), "cudaEventElapsedTime");
    if (s) return s;
  }
  *n_out = n;
  return PKV_OK;
}

}  // extern "C"
