// Shared pieces of the SQ8 leaf kernels (leaf_sq8.cu: 4-warp epilogue and
// rectangular mode; leaf_split.cu: column-split epilogue and the finishing
// kernel): tile geometry, launch parameters, the sorted-bound insertion, the
// candidate-log compaction and the tile table lookup.
#pragma once
#include "common.cuh"

namespace tessa {
namespace leaf {

constexpr uint32_t kBM = 128;          // rows per tile (TMEM lanes)
constexpr uint32_t kBN = 128;          // columns per chunk (MMA N)
constexpr uint32_t kSlab = 128;        // K bytes per TMA box (one 128B swizzle atom)
constexpr uint32_t kMmaK = 32;         // K per tcgen05.mma kind::i8
constexpr uint32_t kMetaSlots = 4;     // chunk metadata ring
constexpr uint32_t kGroup = 32;        // columns per tcgen05.ld
constexpr uint32_t kStashStride = 36;  // floats per lane (16B aligned, conflict-free STS.128)
constexpr uint32_t kLogEntryBytes = 8u;  // (distance bits, global id)
constexpr uint32_t kMaxLogCap = 64;      // entries per row; ranks fit a 64-bit occupancy mask
constexpr uint32_t kSmemLimit = 232448u;  // 227 KiB opt-in per block
constexpr float kTieEps = 2.0e-5f;
constexpr float kMargin = 4.0f * kTieEps;  // zone = [0, theta + kMargin]
constexpr uint32_t kMaxRun = 8;            // longest eps-run checked by tournament

struct Params {
  const float* scales;
  const float* norms;
  const uint32_t* global_ids;
  const uint32_t* members;      // leaf-ordered local ids
  const uint64_t* leaf_starts;
  const uint32_t* leaf_sizes;
  const uint2* tiles;           // (leaf, first row of tile)
  uint32_t num_tiles;
  const uint2* pairs;           // column-split kernel on CTA pairs: (leaf, first row of a 256-row pair)
  uint32_t num_pairs;
  uint32_t num_slabs;
  uint32_t num_bstages;
  uint32_t k;
  uint32_t log_cap;             // log entries per row (<= kMaxLogCap)
  uint64_t resident_rows;
  uint32_t* out_ids;
  float* out_dists;
  uint32_t* err_word;
  uint32_t* fb_count;           // rows handed to the exact fallback
  uint2* fb_list;               // (leaf, row) entries, capacity fb_capacity
  uint32_t fb_capacity;
  uint64_t timeout_ns;
  // rectangular mode only: rows [0, nrows) of the A matrix against columns
  // [0, ncols) of col_codes with per-column scale, norm and tie key
  uint32_t nrows;
  uint32_t ncols;
  const int8_t* col_codes;
  const float* col_scales;
  const float* col_norms;
  const uint32_t* col_keys;
  // column-split kernel only: per-row zone dump for the finishing kernel,
  // rows [dump_row0, dump_row0 + dump_rows) of the leaf-ordered row space
  uint2* dump;           // [dump_d][dump_rows] (distance bits, global id)
  float4* dump_m;        // [8][dump_rows] the row's k smallest, descending, -inf padded to 32
  uint8_t* dump_cnt;     // [dump_rows][2] entries per half, 0xFF = overflow
  uint32_t dump_d;
  uint64_t dump_row0;
  uint64_t dump_rows;
};


__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

__device__ __forceinline__ float fmin3(float a, float b, float c) {
  float r;
  asm("min.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// Sorted array (descending, s[0] = maximum) of the KS smallest values seen.
// Inserting the pair x <= y keeps the KS smallest of s, x and y:
//   new[t] = max(s[t+2], min(s[t+1], y), min(s[t], x))
// (the t-th largest of the merged sequence; s[KS] = s[KS+1] = -inf).  With
// y = +inf it is the single insertion max(s[t+1], min(s[t], x)); values at or
// above s[0] leave s unchanged.  Slots [k, KS) hold -inf sentinels that never
// move, so s[0] is the k-th smallest.  Branch-free: 2 min + 1 three-input max
// per slot.
template <int KS>
__device__ __forceinline__ void topk_insert2(float (&s)[KS], float x, float y) {
  // In place, ascending: slot t reads slots t+1 and t+2 before they change.
#pragma unroll
  for (int t = 0; t < KS; ++t) {
    const float s1 = (t + 1 < KS) ? s[t + 1] : -INFINITY;
    const float s2 = (t + 2 < KS) ? s[t + 2] : -INFINITY;
    s[t] = fmax3(s2, fminf(s1, y), fminf(s[t], x));
  }
}

// Take the next two marked columns (bit 31 - column, highest first) out of
// `mask`; a missing one gets h = false and a harmless in-range index.
__device__ __forceinline__ void next_pair(uint32_t& mask, bool& h0, uint32_t& c0, bool& h1, uint32_t& c1) {
  h0 = mask != 0u;
  c0 = h0 ? __clz(mask) : 0u;
  mask &= ~(h0 ? (0x80000000u >> c0) : 0u);
  h1 = mask != 0u;
  c1 = h1 ? __clz(mask) : 0u;
  mask &= ~(h1 ? (0x80000000u >> c1) : 0u);
}

// Keep the log entries of `row` with distance <= thr, in place.  Entries are
// read eight at a time (all loads before any store of the batch: the write
// index never passes the read index, so the batch is intact).
__device__ __forceinline__ uint32_t log_compact(uint2* log, uint32_t row, uint32_t cnt, float thr) {
  uint32_t j = 0;
  for (uint32_t e0 = 0; e0 < cnt; e0 += 8) {
    uint2 v[8];
#pragma unroll
    for (uint32_t u = 0; u < 8; ++u) v[u] = (e0 + u < cnt) ? log[(e0 + u) * kBM + row] : make_uint2(0x7f800000u, 0u);
#pragma unroll
    for (uint32_t u = 0; u < 8; ++u) {
      if (e0 + u < cnt && __uint_as_float(v[u].x) <= thr) {
        log[j * kBM + row] = v[u];
        ++j;
      }
    }
  }
  return j;
}

// Work item `tile`: (leaf, first row) from the tile table, or in rectangular
// mode (0, 128 * tile) over the whole row matrix.
template <bool RECT>
__device__ __forceinline__ void tile_span(const Params& p, uint32_t tile, uint2& t, uint64_t& start, uint32_t& rows,
                                          uint32_t& cols) {
  if constexpr (RECT) {
    t = make_uint2(0u, tile * kBM);
    start = 0;
    rows = p.nrows;
    cols = p.ncols;
  } else {
    t = p.tiles[tile];
    start = p.leaf_starts[t.x];
    rows = p.leaf_sizes[t.x];
    cols = rows;
  }
}

}  // namespace leaf
}  // namespace tessa
