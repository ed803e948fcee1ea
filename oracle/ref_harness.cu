// Launch harness for the reference's own CUDA kernels (test infrastructure).
//
// The reference (Rust) compiles GPU_PERSISTENT_SUBTREE_KERNEL_SRC with NVRTC
// and launches two of its kernels from TessaCudaReplaySession
// (shear-core/src/algorithm/pipnn/compute_backend.rs:34597-35230):
//   * gpu_tessa_assignment_replay      -- launch_assignment, CB:34971-35024;
//   * gpu_persistent_subtree_topk_only -- launch_leaf,       CB:35026-35157.
// This file includes the extracted kernel text (oracle/_ref/, made by
// extract_ref_kernels.py, never committed) and launches the same kernels with
// the same argument lists, counter clears and launch shapes, from host buffers.
// It is compiled twice, as the reference compiles two modules:
//   REF_HARNESS_ASSIGN -- no feature macros (CB:34676-34689);
//   REF_HARNESS_LEAF   -- GPU_PERSISTENT_LEAF_DCO_ENABLE=1 and
//                         GPU_PERSISTENT_LEAF_SQ_INT8_WMMA_ENABLE=1
//                         (persistent_topk_only_function(.., true, true, ..),
//                         CB:34693-34695, options CB:22377-22384).
// Only tests/ and bench.py's reference legs load the libraries built from it.
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>
#include <chrono>
#include <thread>
#include <vector>

#include "_ref/ref_persistent_subtree.cu"

namespace {

constexpr unsigned kCounterWords = 159;        // GPU_QUEUE_COUNTER_WORDS, CB:274
constexpr unsigned kDiagWords = 24;            // GPU_PERSISTENT_TOPK_WMMA_DIAG_WORDS, CB:480
constexpr unsigned kMaxGridBlocks = 128;       // GPU_PERSISTENT_MAX_GRID_BLOCKS, CB:373
constexpr unsigned kLargeTileRows = 16;        // GPU_PERSISTENT_LARGE_TILE_ROWS, CB:288
constexpr unsigned kLeafTileRows = 128;        // GPU_PERSISTENT_LEAF_TILE_ROWS, CB:391
constexpr double kHostWaitSeconds = 600.0;

thread_local char g_err[512];

int fail(const char* what, cudaError_t e) {
  snprintf(g_err, sizeof g_err, "%s: %s", what, cudaGetErrorString(e));
  return -1;
}

struct DevBuf {
  void* p = nullptr;
  ~DevBuf() {
    if (p) cudaFree(p);
  }
};

#define UPLOAD(buf, src, bytes)                                                     \
  do {                                                                              \
    size_t nb__ = (bytes) ? (bytes) : 16;                                           \
    cudaError_t e__ = cudaMalloc(&(buf).p, nb__);                                   \
    if (e__ != cudaSuccess) return fail("cudaMalloc " #buf, e__);                   \
    if ((src) && (bytes)) {                                                         \
      e__ = cudaMemcpy((buf).p, (src), (bytes), cudaMemcpyHostToDevice);            \
      if (e__ != cudaSuccess) return fail("upload " #buf, e__);                     \
    } else {                                                                        \
      cudaMemset((buf).p, 0, nb__);                                                 \
    }                                                                               \
  } while (0)

// Waits for the launch with a host deadline; the kernels' own loops end once
// the claimed queue is drained (every CTA is co-resident, checked before the
// launch), so the deadline only turns an unexpected stall into an error.
int wait_done(cudaEvent_t done) {
  auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    cudaError_t q = cudaEventQuery(done);
    if (q == cudaSuccess) return 0;
    if (q != cudaErrorNotReady) return fail("kernel", q);
    double s = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if (s > kHostWaitSeconds) {
      snprintf(g_err, sizeof g_err, "reference kernel still running after %.0f s", s);
      return -2;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(200));
  }
}

}  // namespace

extern "C" const char* ref_last_error(void) { return g_err; }

#ifdef REF_HARNESS_LEAF
// One leaf replay through gpu_persistent_subtree_topk_only with the SQ8
// executor `executor` (1 = DP4A scalar filter, 2 = s8 WMMA filter), staged
// column tasks for leaves above 512 rows exactly as tessa_leaf_queue builds
// them (CB:35193-35230).  Outputs are rows x k at member_offset * k.
// `repeats` launches run back to back (outputs and counters cleared before
// each, as run_mode does); ms_out gets the mean kernel time of the launches.
extern "C" int ref_leaf_replay(const float* x, const uint32_t* gids, const float* raw_norms,
                               const int8_t* codes, const float* scales, const float* sq8_norms,
                               uint32_t resident_rows, uint32_t dim, uint32_t padded_dim,
                               const uint32_t* leaf_members, uint32_t leaf_rows,
                               const uint64_t* leaf_starts, const uint64_t* leaf_sizes,
                               uint32_t leaf_count, uint32_t k, uint32_t executor, int staged,
                               int repeats, uint32_t* out_ids, float* out_dists,
                               uint64_t* counters_out, float* ms_out) {
  g_err[0] = 0;
  if (executor != 1 && executor != 2) {
    snprintf(g_err, sizeof g_err, "leaf executor must be 1 (DP4A) or 2 (WMMA)");
    return -3;
  }
  // tessa_leaf_queue (CB:35193-35230): 8 words per (leaf, 128-row tile, column task).
  std::vector<uint32_t> queue;
  size_t raw_tasks = 0;
  for (uint32_t leaf = 0; leaf < leaf_count; ++leaf) {
    uint64_t off = leaf_starts[leaf], cnt = leaf_sizes[leaf];
    uint64_t tiles = (cnt + kLeafTileRows - 1) / kLeafTileRows;
    raw_tasks += tiles;
    uint64_t col_tasks = (staged && cnt > 512) ? (cnt + 127) / 128 : 1;
    for (uint64_t t = 0; t < tiles; ++t) {
      uint64_t to = t * kLeafTileRows;
      uint64_t tr = cnt - to < kLeafTileRows ? cnt - to : kLeafTileRows;
      for (uint64_t c = 0; c < col_tasks; ++c) {
        uint64_t cb = col_tasks == 1 ? 0 : c * 128;
        uint64_t cc = col_tasks == 1 ? cnt : (cnt - cb < 128 ? cnt - cb : 128);
        uint32_t w[8] = {(uint32_t)off, (uint32_t)cnt, leaf, (uint32_t)to, (uint32_t)tr, 1u,
                         (uint32_t)cb, (uint32_t)cc};
        queue.insert(queue.end(), w, w + 8);
      }
    }
  }
  size_t tasks = queue.size() / 8;
  size_t max_tasks = tasks > raw_tasks ? tasks : raw_tasks;
  if (leaf_count > max_tasks) max_tasks = leaf_count;
  size_t out_len = (size_t)leaf_rows * k;

  DevBuf d_x, d_g, d_rn, d_c, d_s, d_n, d_q, d_m, d_st, d_sz, d_ids, d_d, d_lock, d_cnt, d_diag;
  UPLOAD(d_x, x, (size_t)resident_rows * dim * 4);
  UPLOAD(d_g, gids, (size_t)resident_rows * 4);
  UPLOAD(d_rn, raw_norms, (size_t)resident_rows * 4);
  UPLOAD(d_c, codes, (size_t)resident_rows * padded_dim);
  UPLOAD(d_s, scales, (size_t)resident_rows * 4);
  UPLOAD(d_n, sq8_norms, (size_t)resident_rows * 4);
  UPLOAD(d_q, queue.data(), queue.size() * 4);
  UPLOAD(d_m, leaf_members, (size_t)leaf_rows * 4);
  UPLOAD(d_st, leaf_starts, (size_t)leaf_count * 8);
  UPLOAD(d_sz, leaf_sizes, (size_t)leaf_count * 8);
  UPLOAD(d_ids, (const void*)nullptr, out_len * 4);
  UPLOAD(d_d, (const void*)nullptr, out_len * 4);
  UPLOAD(d_lock, (const void*)nullptr, (size_t)leaf_rows * 4);
  UPLOAD(d_cnt, (const void*)nullptr, kCounterWords * 8);
  UPLOAD(d_diag, (const void*)nullptr, kDiagWords * 8);

  int dev = 0, sms = 0, per_sm = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gpu_persistent_subtree_topk_only, 256, 0);
  if (e != cudaSuccess) return fail("occupancy", e);
  unsigned grid = (unsigned)(sms < 1 ? 1 : sms);
  if (grid > kMaxGridBlocks) grid = kMaxGridBlocks;  // persistent_subtree_runtime_grid_block_cap
  if ((long)per_sm * sms < (long)grid) {
    snprintf(g_err, sizeof g_err, "persistent grid %u not co-resident (%d per SM x %d SMs)", grid, per_sm, sms);
    return -4;
  }

  std::vector<uint32_t> clear_ids(out_len, 0xffffffffu);
  std::vector<float> clear_d(out_len, 3.402823466e38f);
  cudaEvent_t ev0, ev1;
  cudaEventCreate(&ev0);
  cudaEventCreate(&ev1);
  float total_ms = 0.0f;
  int rc = 0;
  const unsigned zero = 0u;
  const float sigma = 3.0f;
  const unsigned topk_operator = 3u;      // GPU_PERSISTENT_TOPK_OPERATOR_WMMA_TF32 (SQ8 modes)
  const unsigned leaf_dco_mode = 3u;      // GPU_PERSISTENT_LEAF_DCO_WMMA_FILTER
  const unsigned rerank = 1u;             // GPU_PERSISTENT_LEAF_DCO_RERANK_NONE
  const unsigned distance_source = 2u;    // GPU_PERSISTENT_DISTANCE_SOURCE_SQ_INT8
  const unsigned sq8_leaf_mode = 0u;      // GPU_PERSISTENT_SQ8_LEAF_MODE_STAGED
  const unsigned code_layout = 0u;
  const unsigned max_leaf_count = (unsigned)max_tasks;
  const unsigned long long task_count = tasks;
  for (int it = 0; it < (repeats < 1 ? 1 : repeats) && rc == 0; ++it) {
    // run_mode's clears (CB:34860-34889).
    if ((e = cudaMemcpy(d_ids.p, clear_ids.data(), out_len * 4, cudaMemcpyHostToDevice)) != cudaSuccess ||
        (e = cudaMemcpy(d_d.p, clear_d.data(), out_len * 4, cudaMemcpyHostToDevice)) != cudaSuccess ||
        (e = cudaMemset(d_lock.p, 0, (size_t)leaf_rows * 4)) != cudaSuccess ||
        (e = cudaMemset(d_cnt.p, 0, kCounterWords * 8)) != cudaSuccess) {
      rc = fail("clear", e);
      break;
    }
    cudaEventRecord(ev0);
    gpu_persistent_subtree_topk_only<<<grid, 256>>>(
        (const float*)d_x.p, (const unsigned*)d_g.p, (const float*)d_n.p,
        (const float*)d_rn.p, (const float*)d_rn.p, (const float*)d_rn.p, (const float*)d_rn.p,
        (const signed char*)d_c.p, (const float*)d_s.p, (const float*)d_n.p,
        padded_dim, padded_dim, code_layout,
        (const unsigned char*)nullptr, (const unsigned char*)nullptr,
        (const float*)d_rn.p, (const float*)d_rn.p,
        zero, zero, zero, zero, zero,
        (const unsigned*)d_q.p, (const unsigned*)d_m.p,
        (const unsigned long long*)d_st.p, (const unsigned long long*)d_sz.p,
        (unsigned*)d_ids.p, (float*)d_d.p, (unsigned*)d_lock.p, (unsigned long long*)d_cnt.p,
        resident_rows, dim, k, max_leaf_count, leaf_rows, leaf_rows, leaf_count, task_count,
        topk_operator, leaf_dco_mode, rerank, zero, k, zero, zero, zero, zero, sigma,
        distance_source, sq8_leaf_mode, executor, (unsigned long long*)d_diag.p);
    if ((e = cudaGetLastError()) != cudaSuccess) {
      rc = fail("leaf launch", e);
      break;
    }
    cudaEventRecord(ev1);
    rc = wait_done(ev1);
    if (rc == 0) {
      float ms = 0.0f;
      cudaEventElapsedTime(&ms, ev0, ev1);
      total_ms += ms;
    }
  }
  if (rc == 0) {
    if ((e = cudaMemcpy(out_ids, d_ids.p, out_len * 4, cudaMemcpyDeviceToHost)) != cudaSuccess ||
        (e = cudaMemcpy(out_dists, d_d.p, out_len * 4, cudaMemcpyDeviceToHost)) != cudaSuccess ||
        (e = cudaMemcpy(counters_out, d_cnt.p, kCounterWords * 8, cudaMemcpyDeviceToHost)) != cudaSuccess)
      rc = fail("download", e);
    *ms_out = total_ms / (float)(repeats < 1 ? 1 : repeats);
  }
  cudaEventDestroy(ev0);
  cudaEventDestroy(ev1);
  return rc;
}
#endif  // REF_HARNESS_LEAF

#ifdef REF_HARNESS_ASSIGN
// One assignment replay through gpu_tessa_assignment_replay with executor
// 0 (FP32 SIMT), 1 (TF32 WMMA), 2 (SQ8 DP4A) or 3 (SQ8 WMMA), work items of
// `ticket_batch` 16-row tiles (tessa_assignment_work_device, CB:35159-35191).
extern "C" int ref_assign_replay(const float* x, const uint32_t* gids, const float* raw_norms,
                                 const int8_t* codes, const float* scales, const float* sq8_norms,
                                 uint32_t resident_rows, uint32_t dim, uint32_t padded_dim,
                                 const uint32_t* members, uint32_t member_len,
                                 const uint32_t* leaders, uint32_t leader_len,
                                 const uint32_t* t_moff, const uint32_t* t_mcnt,
                                 const uint32_t* t_loff, const uint32_t* t_lcnt,
                                 const uint32_t* t_rh, const uint64_t* t_out, uint32_t task_count,
                                 uint64_t output_len, uint32_t executor, uint32_t ticket_batch,
                                 int repeats, uint32_t* out_ids, float* out_dists,
                                 uint64_t* counters_out, float* ms_out) {
  g_err[0] = 0;
  std::vector<uint32_t> w_task, w_begin, w_count;
  for (uint32_t t = 0; t < task_count; ++t) {
    uint32_t tiles = (t_mcnt[t] + kLargeTileRows - 1) / kLargeTileRows;
    for (uint32_t b = 0; b < tiles; b += ticket_batch) {
      w_task.push_back(t);
      w_begin.push_back(b);
      w_count.push_back(tiles - b < ticket_batch ? tiles - b : ticket_batch);
    }
  }
  uint32_t work_count = (uint32_t)w_task.size();
  DevBuf d_x, d_g, d_rn, d_c, d_s, d_n, d_mem, d_lead, d_mo, d_mc, d_lo, d_lc, d_rh, d_to, d_wt, d_wb, d_wc,
      d_large, d_best, d_ids, d_d, d_cnt;
  UPLOAD(d_x, x, (size_t)resident_rows * dim * 4);
  UPLOAD(d_g, gids, (size_t)resident_rows * 4);
  UPLOAD(d_rn, raw_norms, (size_t)resident_rows * 4);
  UPLOAD(d_c, codes, (size_t)resident_rows * padded_dim);
  UPLOAD(d_s, scales, (size_t)resident_rows * 4);
  UPLOAD(d_n, sq8_norms, (size_t)resident_rows * 4);
  UPLOAD(d_mem, members, (size_t)member_len * 4);
  UPLOAD(d_lead, leaders, (size_t)leader_len * 4);
  UPLOAD(d_mo, t_moff, (size_t)task_count * 4);
  UPLOAD(d_mc, t_mcnt, (size_t)task_count * 4);
  UPLOAD(d_lo, t_loff, (size_t)task_count * 4);
  UPLOAD(d_lc, t_lcnt, (size_t)task_count * 4);
  UPLOAD(d_rh, t_rh, (size_t)task_count * 4);
  UPLOAD(d_to, t_out, (size_t)task_count * 8);
  UPLOAD(d_wt, w_task.data(), (size_t)work_count * 4);
  UPLOAD(d_wb, w_begin.data(), (size_t)work_count * 4);
  UPLOAD(d_wc, w_count.data(), (size_t)work_count * 4);
  UPLOAD(d_large, (const void*)nullptr, (size_t)member_len * 4);
  UPLOAD(d_best, (const void*)nullptr, (size_t)member_len * 16);
  UPLOAD(d_ids, (const void*)nullptr, output_len * 4);
  UPLOAD(d_d, (const void*)nullptr, output_len * 4);
  UPLOAD(d_cnt, (const void*)nullptr, kCounterWords * 8);

  std::vector<uint32_t> clear_ids(output_len, 0xffffffffu);
  std::vector<float> clear_d(output_len, 3.402823466e38f);
  std::vector<uint64_t> counters(kCounterWords, 0);
  counters[21] = resident_rows;  // run_mode, CB:34849
  cudaEvent_t ev0, ev1;
  cudaEventCreate(&ev0);
  cudaEventCreate(&ev1);
  cudaError_t e;
  float total_ms = 0.0f;
  int rc = 0;
  for (int it = 0; it < (repeats < 1 ? 1 : repeats) && rc == 0; ++it) {
    if ((e = cudaMemcpy(d_ids.p, clear_ids.data(), output_len * 4, cudaMemcpyHostToDevice)) != cudaSuccess ||
        (e = cudaMemcpy(d_d.p, clear_d.data(), output_len * 4, cudaMemcpyHostToDevice)) != cudaSuccess ||
        (e = cudaMemset(d_large.p, 0xff, (size_t)member_len * 4)) != cudaSuccess ||
        (e = cudaMemset(d_best.p, 0xff, (size_t)member_len * 16)) != cudaSuccess ||
        (e = cudaMemcpy(d_cnt.p, counters.data(), kCounterWords * 8, cudaMemcpyHostToDevice)) != cudaSuccess) {
      rc = fail("clear", e);
      break;
    }
    cudaEventRecord(ev0);
    if (work_count > 0) {
      gpu_tessa_assignment_replay<<<work_count, 256>>>(
          (const float*)d_x.p, (const unsigned*)d_g.p, (const float*)d_rn.p, (const signed char*)d_c.p,
          (const float*)d_s.p, (const float*)d_n.p, resident_rows, dim, padded_dim,
          (const unsigned*)d_mem.p, (const unsigned*)d_lead.p, (const unsigned*)d_mo.p,
          (const unsigned*)d_mc.p, (const unsigned*)d_lo.p, (const unsigned*)d_lc.p,
          (const unsigned*)d_rh.p, (const unsigned long long*)d_to.p, task_count,
          (const unsigned*)d_wt.p, (const unsigned*)d_wb.p, (const unsigned*)d_wc.p, work_count, executor,
          (unsigned*)d_large.p, (unsigned*)d_best.p, (unsigned*)d_ids.p, (float*)d_d.p,
          (unsigned long long*)d_cnt.p);
      if ((e = cudaGetLastError()) != cudaSuccess) {
        rc = fail("assignment launch", e);
        break;
      }
    }
    cudaEventRecord(ev1);
    rc = wait_done(ev1);
    if (rc == 0) {
      float ms = 0.0f;
      cudaEventElapsedTime(&ms, ev0, ev1);
      total_ms += ms;
    }
  }
  if (rc == 0) {
    if ((e = cudaMemcpy(out_ids, d_ids.p, output_len * 4, cudaMemcpyDeviceToHost)) != cudaSuccess ||
        (e = cudaMemcpy(out_dists, d_d.p, output_len * 4, cudaMemcpyDeviceToHost)) != cudaSuccess ||
        (e = cudaMemcpy(counters_out, d_cnt.p, kCounterWords * 8, cudaMemcpyDeviceToHost)) != cudaSuccess)
      rc = fail("download", e);
    *ms_out = total_ms / (float)(repeats < 1 ? 1 : repeats);
  }
  cudaEventDestroy(ev0);
  cudaEventDestroy(ev1);
  return rc;
}
#endif  // REF_HARNESS_ASSIGN
