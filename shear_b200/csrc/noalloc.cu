// tessa_leaf_topk_sq8_noalloc: the SQ8 leaf top-k for callers that cannot
// allocate device memory.
//
// Who needs it: a host whose allocator already owns the whole device (a build
// that reserves its GPU workspace up front and hands out sub-buffers), code on
// a latency-critical thread where cudaMalloc/cudaFree -- which can synchronise
// the device -- are not allowed, and embedders that must fix their memory
// footprint when the library is loaded.  tessa_leaf_topk_sq8 cannot serve them:
// it needs a context and grows device scratch on demand (the leaf-ordered copy
// of the codes, the tile table, the exact-fallback row list, the error word).
//
// This entry point keeps that scratch in one file-scope __device__ array of
// TESSA_NOALLOC_SCRATCH_BYTES (64 MiB) instead.  Every GPU that loads the
// library holds the array until the process exits.  Host code must not use the
// array's symbol as a device address: the first call on each device (with that
// device current) resolves the real address with cudaGetSymbolAddress and
// caches it, so that first call should be made before any stream capture.
// The cached address belongs to the device's primary context: after
// cudaDeviceReset (or anything else that destroys that context) it is stale,
// and this entry point must not be called again in that process.
// All calls share the array and a call leaves its contents behind; calls whose
// GPU work overlaps (same device, different streams, or different host threads)
// race on it and must be serialised by the caller.  The call allocates nothing:
// no cudaMalloc, cudaFree, cudaMallocAsync, context or stream creation, and no
// host heap allocation (host-side staging goes through fixed stack buffers).
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace {

constexpr size_t kScratchBytes = TESSA_NOALLOC_SCRATCH_BYTES;
constexpr size_t kAlign = 256;
constexpr int kMaxDevices = 64;
constexpr uint64_t kTimeoutNs = 2000000000ull;
constexpr uint32_t kTileRows = 128;   // rows per leaf tile of the leaf kernel
constexpr int kStage = 2048;          // host stack staging entries per copy

__device__ __align__(256) unsigned char g_leaf_noalloc_scratch[kScratchBytes];

std::mutex g_setup_mu;
void* g_scratch_addr[kMaxDevices];  // device address of g_leaf_noalloc_scratch, per device
int g_sm_count[kMaxDevices];

size_t round_up(size_t v) { return (v + kAlign - 1) / kAlign * kAlign; }

int err(int code, const char* fmt, ...) {
  char buf[384];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  return tessa::set_last_error(code, buf);
}

int cuda_err(cudaError_t e, const char* what) {
  return err(e == cudaErrorMemoryAllocation ? TESSA_ERR_OOM : TESSA_ERR_CUDA, "%s: %s", what,
             cudaGetErrorString(e));
}

// Once per device, with that device current: resolve the scratch address.
int setup_device(int dev, void** addr, int* sms) {
  if (dev < 0 || dev >= kMaxDevices) return err(TESSA_ERR_UNSUPPORTED, "device %d beyond %d", dev, kMaxDevices);
  std::lock_guard<std::mutex> lock(g_setup_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_leaf_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) return cuda_err(e, "cudaGetSymbolAddress(leaf scratch)");
    int n = 0;
    e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_err(e, "cudaDeviceGetAttribute(multiProcessorCount)");
    g_sm_count[dev] = n;
    g_scratch_addr[dev] = p;
  }
  *addr = g_scratch_addr[dev];
  *sms = g_sm_count[dev];
  return TESSA_OK;
}

}  // namespace

extern "C" int tessa_leaf_topk_sq8_noalloc(const tessa_leaf_args* a, void* stream) {
  using namespace tessa;
  if (!a) return err(TESSA_ERR_INVALID_ARG, "null leaf args");
  if (a->k == 0 || a->k > TESSA_MAX_LEAF_K)
    return err(TESSA_ERR_INVALID_ARG, "leaf k=%u outside 1..%d", a->k, TESSA_MAX_LEAF_K);
  if (a->padded_dim == 0 || a->padded_dim % 16 != 0)
    return err(TESSA_ERR_INVALID_ARG, "padded_dim=%u must be a positive multiple of 16", a->padded_dim);
  if (a->padded_dim > TESSA_MAX_PADDED_DIM || leaf_num_bstages(a->padded_dim) == 0)
    return err(TESSA_ERR_UNSUPPORTED, "padded_dim=%u above the supported %d", a->padded_dim, TESSA_MAX_PADDED_DIM);
  if (a->leaf_count && (!a->leaf_starts || !a->leaf_sizes)) return err(TESSA_ERR_INVALID_ARG, "null leaf layout");
  if (a->leaf_rows && (!a->leaf_members || !a->codes || !a->scales || !a->norms || !a->global_ids ||
                       !a->topk_ids || !a->topk_dists))
    return err(TESSA_ERR_INVALID_ARG, "null leaf data pointer");
  if (a->leaf_rows > 0x7fffffffull) return err(TESSA_ERR_UNSUPPORTED, "more than 2^31 leaf member rows");
  if (a->resident_rows > 0xffffffffull) return err(TESSA_ERR_UNSUPPORTED, "more than 2^32 resident rows");

  // Tile count and layout checks (no host allocation: one pass over the layout).
  uint64_t num_tiles = 0;
  for (uint64_t l = 0; l < a->leaf_count; ++l) {
    uint64_t st = a->leaf_starts[l], sz = a->leaf_sizes[l];
    if (sz > kMaxLeafRows)
      return err(TESSA_ERR_UNSUPPORTED, "leaf %llu has %llu rows; at most %llu are supported", (unsigned long long)l,
                 (unsigned long long)sz, (unsigned long long)kMaxLeafRows);
    if (st > a->leaf_rows || sz > a->leaf_rows - st)
      return err(TESSA_ERR_INVALID_ARG, "leaf %llu [start %llu, size %llu] outside %llu member rows",
                 (unsigned long long)l, (unsigned long long)st, (unsigned long long)sz,
                 (unsigned long long)a->leaf_rows);
    num_tiles += (sz + kTileRows - 1) / kTileRows;
  }

  // Scratch layout inside the static array.
  const bool gather = a->leaf_ordered_codes == nullptr;
  size_t off_err = 0;
  size_t off_starts = round_up(off_err + 4);
  size_t off_sizes = round_up(off_starts + a->leaf_count * 8);
  size_t off_tiles = round_up(off_sizes + a->leaf_count * 4);
  size_t off_fb = round_up(off_tiles + num_tiles * 8);
  size_t off_codes = round_up(off_fb + 16 + (size_t)a->leaf_rows * 8);
  size_t need = gather ? off_codes + (size_t)a->leaf_rows * a->padded_dim : off_codes;
  if (need > kScratchBytes)
    return err(TESSA_ERR_UNSUPPORTED,
               "tessa_leaf_topk_sq8_noalloc: this batch needs %zu bytes of scratch, above the static %zu-byte "
               "limit (pass leaf_ordered_codes, split the batch, or use tessa_leaf_topk_sq8)",
               need, kScratchBytes);

  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_err(e, "cudaGetDevice");
  void* base = nullptr;
  int sms = 0;
  int r = setup_device(dev, &base, &sms);
  if (r != TESSA_OK) return r;
  if (num_tiles == 0) return TESSA_OK;
  unsigned char* s = static_cast<unsigned char*>(base);
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  // Zero the error word, upload the layout and the tile table through stack
  // staging (pageable copies return once the source has been staged).
  if ((e = cudaMemsetAsync(s + off_err, 0, 4, st)) != cudaSuccess) return cuda_err(e, "clear error word");
  if (a->leaf_count &&
      (e = cudaMemcpyAsync(s + off_starts, a->leaf_starts, a->leaf_count * 8, cudaMemcpyHostToDevice, st)) !=
          cudaSuccess)
    return cuda_err(e, "upload leaf starts");
  uint32_t sz_stage[kStage];
  for (uint64_t l0 = 0; l0 < a->leaf_count; l0 += kStage) {
    uint64_t n = a->leaf_count - l0 < (uint64_t)kStage ? a->leaf_count - l0 : (uint64_t)kStage;
    for (uint64_t i = 0; i < n; ++i) sz_stage[i] = (uint32_t)a->leaf_sizes[l0 + i];
    if ((e = cudaMemcpyAsync(s + off_sizes + l0 * 4, sz_stage, n * 4, cudaMemcpyHostToDevice, st)) != cudaSuccess)
      return cuda_err(e, "upload leaf sizes");
  }
  uint2 tile_stage[kStage];
  uint64_t t_out = 0;
  int t_fill = 0;
  for (uint64_t l = 0; l < a->leaf_count; ++l) {
    for (uint64_t r0 = 0; r0 < a->leaf_sizes[l]; r0 += kTileRows) {
      tile_stage[t_fill++] = make_uint2((uint32_t)l, (uint32_t)r0);
      if (t_fill == kStage) {
        if ((e = cudaMemcpyAsync(s + off_tiles + t_out * 8, tile_stage, (size_t)t_fill * 8, cudaMemcpyHostToDevice,
                                 st)) != cudaSuccess)
          return cuda_err(e, "upload tile table");
        t_out += t_fill;
        t_fill = 0;
      }
    }
  }
  if (t_fill &&
      (e = cudaMemcpyAsync(s + off_tiles + t_out * 8, tile_stage, (size_t)t_fill * 8, cudaMemcpyHostToDevice, st)) !=
          cudaSuccess)
    return cuda_err(e, "upload tile table");

  const int8_t* leaf_codes = a->leaf_ordered_codes;
  if (gather) {
    r = launch_gather_rows(a->codes, a->leaf_members, a->leaf_rows, a->padded_dim, a->resident_rows,
                           reinterpret_cast<int8_t*>(s + off_codes), sms, st);
    if (r != TESSA_OK) return err(r, "gather kernel launch failed (code %d)", r);
    leaf_codes = reinterpret_cast<const int8_t*>(s + off_codes);
  }

  LeafLaunch L;
  L.leaf_codes = leaf_codes;
  L.leaf_rows = a->leaf_rows;
  L.padded_dim = a->padded_dim;
  L.scales = a->scales;
  L.norms = a->norms;
  L.global_ids = a->global_ids;
  L.members = a->leaf_members;
  L.d_leaf_starts = reinterpret_cast<const uint64_t*>(s + off_starts);
  L.d_leaf_sizes = reinterpret_cast<const uint32_t*>(s + off_sizes);
  L.d_tiles = reinterpret_cast<const uint2*>(s + off_tiles);
  L.num_tiles = (uint32_t)num_tiles;
  L.k = a->k;
  L.out_ids = a->topk_ids;
  L.out_dists = a->topk_dists;
  L.d_err = reinterpret_cast<uint32_t*>(s + off_err);
  L.d_fb_count = reinterpret_cast<uint32_t*>(s + off_fb);
  L.d_fb_list = reinterpret_cast<uint2*>(s + off_fb + 16);
  L.fb_capacity = (uint32_t)a->leaf_rows;
  L.resident_rows = a->resident_rows;
  L.timeout_ns = kTimeoutNs;
  L.sm_count = sms;
  r = launch_leaf_topk_sq8(L, st);
  if (r != TESSA_OK) return err(r, "leaf kernel launch failed (code %d)", r);

  uint32_t bits = 0;
  if ((e = cudaMemcpyAsync(&bits, s + off_err, 4, cudaMemcpyDeviceToHost, st)) != cudaSuccess)
    return cuda_err(e, "read error word");
  if ((e = cudaStreamSynchronize(st)) != cudaSuccess) return cuda_err(e, "stream synchronize");
  if (bits & TESSA_DEVERR_TIMEOUT) return err(TESSA_ERR_TIMEOUT, "device wait timed out (0x%x)", bits);
  if (bits & TESSA_DEVERR_BAD_ROW) return err(TESSA_ERR_BAD_ROW, "row id outside resident rows (0x%x)", bits);
  if (bits) return err(TESSA_ERR_BAD_TASK, "device error bits 0x%x", bits);
  return TESSA_OK;
}
