// Subtree submissions: partition + leaf top-k of a batch of subtree tasks,
// with the CompactTopKBatch copied into a two-slot pinned ring.
//
// The reference overlaps the GPU's work on one subtree batch with the host's
// scatter of the previous one: submit_owned_quantized_subtree_l2_compact_topk
// (shear-core/src/algorithm/pipnn/compute_backend.rs:3693-3884) hands a batch
// to the engine and returns a submission, and the persistent async D2H ring
// (persistent_async_d2h.rs:4-80, PERSISTENT_ASYNC_D2H_SLOT_COUNT = 2) keeps
// each batch's device and pinned host output slots leased from compute to
// copy to the host consumer's scatter, publishing batches in sequence order.
//
// Here a submission takes one of two slots (Free -> Running -> Ready ->
// Held -> Free), and a worker thread runs it on a private context of the
// same device (its own stream and scratch, so the caller's context stays
// usable meanwhile): tessa_subtree_partition into the slot's leaf arena,
// tessa_leaf_topk_sq8 over its leaves, point ids gathered from the global
// ids, and one copy of rows, ids and distances into the slot's pinned
// buffers.  poll reports a batch once its copy has landed; the view stays
// valid until release.  Jobs run in submission order.
#include <condition_variable>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <deque>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "common.cuh"
#include "kernels.h"

namespace tessa {
namespace submit {

__global__ void point_ids_kernel(const uint32_t* leaf_rows, uint64_t rows, const uint32_t* global_ids,
                                 uint64_t resident_rows, uint32_t* out) {
  for (uint64_t r = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; r < rows; r += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t m = leaf_rows[r];
    out[r] = m < resident_rows ? global_ids[m] : 0xffffffffu;
  }
}

__global__ void fill_kernel(uint32_t* ids, float* dists, uint64_t n) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
    ids[i] = 0xffffffffu;
    dists[i] = INFINITY;
  }
}

enum class State { Free, Running, Ready, Held };

struct Pinned {
  void* p = nullptr;
  size_t bytes = 0;
  bool ensure(size_t need) {
    if (need <= bytes) return true;
    if (p) cudaFreeHost(p);
    p = nullptr;
    bytes = 0;
    if (cudaHostAlloc(&p, need, cudaHostAllocDefault) != cudaSuccess) {
      p = nullptr;
      return false;
    }
    bytes = need;
    return true;
  }
  void release() {
    if (p) cudaFreeHost(p);
    p = nullptr;
    bytes = 0;
  }
};

struct Device {
  void* p = nullptr;
  size_t bytes = 0;
  bool ensure(size_t need) {
    if (need <= bytes) return true;
    if (p) cudaFree(p);
    p = nullptr;
    bytes = 0;
    if (cudaMalloc(&p, need) != cudaSuccess) {
      p = nullptr;
      return false;
    }
    bytes = need;
    return true;
  }
  void release() {
    if (p) cudaFree(p);
    p = nullptr;
    bytes = 0;
  }
};

struct Slot {
  State state = State::Free;
  uint64_t ticket = 0;
  // the request, with its host arrays owned here
  tessa_subtree_request req{};
  std::vector<uint64_t> task_offsets, task_seeds;
  std::vector<uint32_t> task_counts;
  cudaEvent_t inputs_ready = nullptr;  // recorded on the caller's stream at submit
  // outputs
  Device d_rows, d_pids, d_ids, d_dists;
  Pinned h_pids, h_ids, h_dists;
  std::vector<uint64_t> leaf_starts;
  std::vector<uint32_t> leaf_sizes, leaf_tasks;
  tessa_subtree_result result{};
  uint64_t rows = 0, fallback_rows = 0;
  int rc = TESSA_OK;
  std::string message;
};

}  // namespace submit

struct SubmitRing {
  int device = 0;
  tessa_ctx* worker_ctx = nullptr;
  cudaStream_t stream = nullptr;
  submit::Slot slots[2];
  std::deque<int> queue;  // slot indices in submission order
  uint64_t next_ticket = 1;
  bool stop = false;
  std::mutex m;
  std::condition_variable cv;
  std::thread worker;
};

namespace {

using submit::State;

int errf(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  return set_last_error(code, buf);
}

int run_job(SubmitRing* R, submit::Slot& S) {
  using namespace submit;
  const tessa_subtree_args& in = S.req.partition;
  cudaStream_t st = R->stream;
  if (cudaStreamWaitEvent(st, S.inputs_ready, 0) != cudaSuccess)
    return set_last_error(TESSA_ERR_CUDA, "submission: waiting for the caller's stream failed");
  const uint32_t fs = in.fanout_second ? in.fanout_second : 1u;
  uint64_t task_rows = 0;  // the leaf arena holds at most fanout_second rows per task row
  for (uint32_t t = 0; t < in.task_count; ++t) task_rows += S.task_counts[t];
  const uint64_t cap = (uint64_t)fs * task_rows + 16;
  if (!S.d_rows.ensure(cap * 4)) return set_last_error(TESSA_ERR_OOM, "submission: leaf arena allocation failed");
  S.leaf_starts.assign(cap, 0);
  S.leaf_sizes.assign(cap, 0);
  S.leaf_tasks.assign(cap, 0);
  tessa_subtree_args a = in;
  a.leaf_codes = nullptr;  // the slot keeps no leaf-ordered copy
  a.task_offsets = S.task_offsets.data();
  a.task_counts = S.task_counts.data();
  a.task_seeds = S.task_seeds.data();
  a.leaf_rows = reinterpret_cast<uint32_t*>(S.d_rows.p);
  a.leaf_rows_capacity = cap;
  a.leaf_starts = S.leaf_starts.data();
  a.leaf_sizes = S.leaf_sizes.data();
  a.leaf_tasks = S.leaf_tasks.data();
  a.leaf_capacity = cap;
  int rc = tessa_subtree_partition(R->worker_ctx, &a, &S.result, st);
  if (rc != TESSA_OK) return rc;
  const uint64_t rows = S.result.leaf_rows_used, leaves = S.result.leaf_count, k = S.req.k;
  S.rows = rows;
  if (!S.d_pids.ensure(rows * 4 + 4) || !S.d_ids.ensure(rows * k * 4 + 4) || !S.d_dists.ensure(rows * k * 4 + 4))
    return set_last_error(TESSA_ERR_OOM, "submission: output allocation failed");
  if (!S.h_pids.ensure(rows * 4 + 4) || !S.h_ids.ensure(rows * k * 4 + 4) || !S.h_dists.ensure(rows * k * 4 + 4))
    return set_last_error(TESSA_ERR_OOM, "submission: pinned output allocation failed");
  uint32_t* ids = reinterpret_cast<uint32_t*>(S.d_ids.p);
  float* dists = reinterpret_cast<float*>(S.d_dists.p);
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, R->device);
  const unsigned grid = (unsigned)(sms > 0 ? sms * 4 : 148);
  if (rows) {
    fill_kernel<<<grid, 256, 0, st>>>(ids, dists, rows * k);
    point_ids_kernel<<<grid, 256, 0, st>>>(reinterpret_cast<const uint32_t*>(S.d_rows.p), rows,
                                           S.req.global_ids, in.resident_rows,
                                           reinterpret_cast<uint32_t*>(S.d_pids.p));
    if (cudaGetLastError() != cudaSuccess) return set_last_error(TESSA_ERR_CUDA, "submission: launch failed");
  }
  if (leaves) {
    std::vector<uint64_t> sizes(leaves);
    for (uint64_t l = 0; l < leaves; ++l) sizes[l] = S.leaf_sizes[l];
    tessa_leaf_args la{};
    la.codes = in.codes;
    la.scales = in.scales;
    la.norms = in.sq8_norms;
    la.global_ids = S.req.global_ids;
    la.resident_rows = in.resident_rows;
    la.padded_dim = in.padded_dim;
    la.k = (uint32_t)k;
    la.leaf_members = reinterpret_cast<const uint32_t*>(S.d_rows.p);
    la.leaf_starts = S.leaf_starts.data();
    la.leaf_sizes = sizes.data();
    la.leaf_count = leaves;
    la.leaf_rows = rows;
    la.topk_ids = ids;
    la.topk_dists = dists;
    rc = tessa_leaf_topk_sq8(R->worker_ctx, &la, st);
    if (rc != TESSA_OK) return rc;
    tessa_leaf_last_fallback_rows(R->worker_ctx, &S.fallback_rows);
  }
  if (rows) {
    if (cudaMemcpyAsync(S.h_pids.p, S.d_pids.p, rows * 4, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaMemcpyAsync(S.h_ids.p, ids, rows * k * 4, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaMemcpyAsync(S.h_dists.p, dists, rows * k * 4, cudaMemcpyDeviceToHost, st) != cudaSuccess)
      return set_last_error(TESSA_ERR_CUDA, "submission: output copy failed");
  }
  if (cudaStreamSynchronize(st) != cudaSuccess) return set_last_error(TESSA_ERR_CUDA, "submission: stream failed");
  return TESSA_OK;
}

void worker_loop(SubmitRing* R) {
  cudaSetDevice(R->device);
  for (;;) {
    int idx;
    {
      std::unique_lock<std::mutex> lk(R->m);
      R->cv.wait(lk, [&] { return R->stop || !R->queue.empty(); });
      if (R->queue.empty()) return;  // stop requested and nothing left
      idx = R->queue.front();
      R->queue.pop_front();
    }
    submit::Slot& S = R->slots[idx];
    const int rc = run_job(R, S);
    {
      std::lock_guard<std::mutex> lk(R->m);
      S.rc = rc;
      S.message = rc == TESSA_OK ? std::string() : std::string(tessa_last_error_message());
      S.state = State::Ready;
    }
    R->cv.notify_all();
  }
}

submit::Slot* find(SubmitRing* R, uint64_t ticket) {
  for (auto& s : R->slots)
    if (s.state != State::Free && s.ticket == ticket) return &s;
  return nullptr;
}

}  // namespace

int submit_ring_create(int device, SubmitRing** out) {
  *out = nullptr;
  SubmitRing* R = new (std::nothrow) SubmitRing();
  if (!R) return set_last_error(TESSA_ERR_OOM, "submission ring allocation failed");
  R->device = device;
  int rc = tessa_create(device, &R->worker_ctx);
  if (rc == TESSA_OK && cudaStreamCreateWithFlags(&R->stream, cudaStreamNonBlocking) != cudaSuccess)
    rc = set_last_error(TESSA_ERR_CUDA, "submission stream create failed");
  for (auto& s : R->slots)
    if (rc == TESSA_OK && cudaEventCreateWithFlags(&s.inputs_ready, cudaEventDisableTiming) != cudaSuccess)
      rc = set_last_error(TESSA_ERR_CUDA, "submission event create failed");
  if (rc != TESSA_OK) {
    submit_ring_destroy(R);
    return rc;
  }
  R->worker = std::thread(worker_loop, R);
  *out = R;
  return TESSA_OK;
}

void submit_ring_destroy(SubmitRing* R) {
  if (!R) return;
  {
    std::lock_guard<std::mutex> lk(R->m);
    R->stop = true;
  }
  R->cv.notify_all();
  if (R->worker.joinable()) R->worker.join();  // queued jobs finish first (every device wait is bounded)
  cudaSetDevice(R->device);
  for (auto& s : R->slots) {
    s.d_rows.release();
    s.d_pids.release();
    s.d_ids.release();
    s.d_dists.release();
    s.h_pids.release();
    s.h_ids.release();
    s.h_dists.release();
    if (s.inputs_ready) cudaEventDestroy(s.inputs_ready);
  }
  if (R->stream) cudaStreamDestroy(R->stream);
  tessa_destroy(R->worker_ctx);
  delete R;
}

int submit_ring_submit(SubmitRing* R, const tessa_subtree_request* req, uint64_t* ticket, cudaStream_t caller) {
  using namespace submit;
  const tessa_subtree_args& a = req->partition;
  std::lock_guard<std::mutex> lk(R->m);
  Slot* S = nullptr;
  for (auto& s : R->slots)
    if (s.state == State::Free) {
      S = &s;
      break;
    }
  if (!S)
    return set_last_error(TESSA_ERR_AGAIN, "both submission slots are leased: poll and release an earlier ticket");
  if (cudaEventRecord(S->inputs_ready, caller) != cudaSuccess)
    return set_last_error(TESSA_ERR_CUDA, "submission: recording the caller's stream failed");
  S->req = *req;
  S->task_offsets.assign(a.task_offsets, a.task_offsets + a.task_count);
  S->task_counts.assign(a.task_counts, a.task_counts + a.task_count);
  S->task_seeds.assign(a.task_seeds, a.task_seeds + a.task_count);
  S->result = tessa_subtree_result{};
  S->rows = S->fallback_rows = 0;
  S->rc = TESSA_OK;
  S->message.clear();
  S->ticket = R->next_ticket++;
  S->state = State::Running;
  R->queue.push_back((int)(S - R->slots));
  *ticket = S->ticket;
  R->cv.notify_all();
  return TESSA_OK;
}

int submit_ring_poll(SubmitRing* R, uint64_t ticket, int wait, tessa_compact_view* view) {
  using namespace submit;
  std::unique_lock<std::mutex> lk(R->m);
  Slot* S = find(R, ticket);
  if (!S) return errf(TESSA_ERR_INVALID_ARG, "ticket %llu is not leased (never issued or released)",
                      (unsigned long long)ticket);
  if (S->state == State::Running) {
    if (!wait) return errf(TESSA_ERR_AGAIN, "submission %llu still running", (unsigned long long)ticket);
    R->cv.wait(lk, [&] { return S->state != State::Running; });
  }
  if (S->rc != TESSA_OK) {
    const int rc = S->rc;
    const std::string msg = S->message;
    S->state = State::Free;  // a failed batch holds nothing
    return errf(rc, "submission %llu: %s", (unsigned long long)ticket, msg.c_str());
  }
  S->state = State::Held;
  std::memset(view, 0, sizeof(*view));
  view->ticket = ticket;
  view->rows = S->rows;
  view->k = S->req.k;
  view->leaf_count = S->result.leaf_count;
  view->leaf_starts = S->leaf_starts.data();
  view->leaf_sizes = S->leaf_sizes.data();
  view->leaf_tasks = S->leaf_tasks.data();
  view->point_ids = reinterpret_cast<const uint32_t*>(S->h_pids.p);
  view->topk_ids = reinterpret_cast<const uint32_t*>(S->h_ids.p);
  view->topk_dists = reinterpret_cast<const float*>(S->h_dists.p);
  view->partition = S->result;
  view->fallback_rows = S->fallback_rows;
  return TESSA_OK;
}

int submit_ring_release(SubmitRing* R, uint64_t ticket) {
  using namespace submit;
  std::lock_guard<std::mutex> lk(R->m);
  Slot* S = find(R, ticket);
  if (!S || S->state == State::Running)
    return errf(TESSA_ERR_INVALID_ARG, "ticket %llu cannot be released (not leased, or still running)",
                (unsigned long long)ticket);
  S->state = State::Free;
  return TESSA_OK;
}

}  // namespace tessa
