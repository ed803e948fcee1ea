// SQ8 leaf all-pairs evaluation with fused per-row bounded top-k, sm_100a.
//
// Reference semantics (wbh1765091327/SHEAR, CB = shear-core/src/algorithm/
// pipnn/compute_backend.rs):
//   * candidates of row r are the other members of its leaf, taken in
//     ascending member position, skipping columns whose local id equals the
//     row's (CB:9569-9650, CB:10046-10096);
//   * distance = gpu_persistent_sq_int8_l2_from_dot (CB:8987-9002);
//   * each candidate goes through gpu_persistent_insert_topk_candidate_fp32
//     (CB:7229-7259) into a k-slot list initialised to (FLT_MAX, 0xffffffff):
//     "better" = |d1-d2| <= 2e-5 ? id1 < id2 : d1 < d2 (not transitive);
//   * output ids are the candidates' global ids, written at (start + r) * k.
//
// How the result is computed without the reference's sequential insertion:
// Let L be a set of k candidates and "<" the eps/id relation above.  If (a)
// every member of L beats every candidate outside L and (b) "<" restricted to
// L is a strict total order, then sequential insertion in ANY order ends with
// exactly L sorted by "<": an L-candidate always passes the list's tail (which
// holds only non-L candidates or empty slots), is never pushed out (only a
// full list of L-candidates could do it), and stops exactly at its rank
// because "<" is transitive on L.  The epilogue therefore selects, per row and
// in any order, the H = k+4 candidates that are smallest by distance, sorts
// them by (distance, member position), splits them into runs of neighbours
// closer than the tie eps, and checks (a) and (b): every run up to the one
// holding rank k must be a transitive tournament under "<" (always true for
// runs of one or two), and that run must end inside the H (or the H must hold
// every candidate).  Rows that pass are written directly; the rest (~4e-4 of
// rows on random data) are listed and recomputed by leaf_fallback_kernel with
// the reference's exact sequential insertion.
//
// B200 design (one persistent CTA per SM, 192 threads):
//   warp 0      TMA producer: A = 128 leaf rows x padded_dim, resident for the
//               tile; B = 128-column chunks streamed in 128-byte K slabs
//               through a ring of shared-memory stages (SWIZZLE_128B).
//   warp 1      TMEM owner + single-thread tcgen05.mma issuer (kind::i8,
//               M=128, N=128, K=32, int32 accumulators) into four 128-column
//               TMEM buffers, so MMAs run up to three chunks ahead.
//   warps 2..5  epilogue: thread t owns TMEM lane (leaf row) t; per 32
//               columns it computes the exact reference distances, marks the
//               ones below its set's current maximum in a bit mask, stashes the
//               distances in shared memory and then inserts the marked ones
//               into an unsorted H-slot set (six blocks of six slots, block
//               maxima in registers).
// The distance matrix never leaves the SM.
#include "common.cuh"
#include "kernels.h"

namespace tessa {
namespace leaf {

constexpr uint32_t kBM = 128;          // rows per tile (TMEM lanes)
constexpr uint32_t kBN = 128;          // columns per chunk (MMA N)
constexpr uint32_t kSlab = 128;        // K bytes per TMA box (one 128B swizzle atom)
constexpr uint32_t kMmaK = 32;         // K per tcgen05.mma kind::i8
constexpr uint32_t kThreads = 192;
constexpr uint32_t kEpiThreads = 128;
constexpr uint32_t kAccBufs = 4;
constexpr uint32_t kTmemCols = kAccBufs * kBN;  // 512
constexpr uint32_t kASlabBytes = kBM * kSlab;   // 16 KiB
constexpr uint32_t kBStageBytes = kBN * kSlab;  // 16 KiB
constexpr uint32_t kGroup = 32;                 // columns per tcgen05.ld
constexpr uint32_t kGroups = kBN / kGroup;
constexpr uint32_t kMaxBStages = 8;
constexpr uint32_t kSetSlots = 36;              // H <= k + 4 <= 36
constexpr uint32_t kBlk = 6;                    // slots per block
constexpr uint32_t kNBlk = kSetSlots / kBlk;    // blocks
constexpr uint32_t kExtra = 4;                  // H = k + kExtra
constexpr uint32_t kMetaBytes = 2u * kBN * 16u;           // 2 chunk buffers of (s, n, lid, -)
constexpr uint32_t kStashBytes = 4u * kGroup * 32u * 4u;  // per epilogue warp: 32 x 32 floats
constexpr uint32_t kSetDBytes = kSetSlots * kBM * 4u;
constexpr uint32_t kSetJBytes = kSetSlots * kBM * 2u;
constexpr uint32_t kBarBytes = 512u;
constexpr uint32_t kSmemLimit = 232448u;  // 227 KiB opt-in per block
constexpr float kTieEps = 2.0e-5f;

struct Params {
  const float* scales;
  const float* norms;
  const uint32_t* global_ids;
  const uint32_t* members;      // leaf-ordered local ids
  const uint64_t* leaf_starts;
  const uint32_t* leaf_sizes;
  const uint2* tiles;           // (leaf, first row of tile)
  uint32_t num_tiles;
  uint32_t num_slabs;
  uint32_t num_bstages;
  uint32_t k;
  uint32_t h;                   // set size H = min(k + 4, 36)
  uint64_t resident_rows;
  uint32_t* out_ids;
  float* out_dists;
  uint32_t* err_word;
  uint32_t* fb_count;           // rows handed to the exact fallback
  uint2* fb_list;               // (leaf, row) entries, capacity fb_capacity
  uint32_t fb_capacity;
  uint64_t timeout_ns;
};

struct Smem {
  uint8_t* a;
  uint8_t* b;
  uint4* meta;
  float* stash;
  float* set_d;     // [slot][row]
  uint16_t* set_j;  // [slot][row]
  uint64_t* a_full;
  uint64_t* a_empty;
  uint64_t* b_full;
  uint64_t* b_empty;
  uint64_t* t_full;
  uint64_t* t_empty;
  uint64_t* mma_done;
  uint32_t* tmem_slot;
  uint32_t* abort_flag;
  volatile uint32_t* epi_stop;
};

__host__ __device__ inline uint32_t smem_bytes(uint32_t num_slabs, uint32_t num_bstages) {
  return 1024u + num_slabs * kASlabBytes + num_bstages * kBStageBytes + kMetaBytes + kStashBytes + kSetDBytes +
         kSetJBytes + kBarBytes;
}

__device__ __forceinline__ Smem carve(uint8_t* raw, uint32_t num_slabs, uint32_t num_bstages) {
  uintptr_t base = (reinterpret_cast<uintptr_t>(raw) + 1023u) & ~uintptr_t(1023u);
  uint8_t* p = reinterpret_cast<uint8_t*>(base);
  Smem s;
  s.a = p;
  p += num_slabs * kASlabBytes;
  s.b = p;
  p += num_bstages * kBStageBytes;
  s.meta = reinterpret_cast<uint4*>(p);
  p += kMetaBytes;
  s.stash = reinterpret_cast<float*>(p);
  p += kStashBytes;
  s.set_d = reinterpret_cast<float*>(p);
  p += kSetDBytes;
  s.set_j = reinterpret_cast<uint16_t*>(p);
  p += kSetJBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(p);
  s.a_full = bars + 0;
  s.a_empty = bars + 1;
  s.b_full = bars + 2;
  s.b_empty = bars + 2 + kMaxBStages;
  s.t_full = bars + 2 + 2 * kMaxBStages;
  s.t_empty = s.t_full + kAccBufs;
  s.mma_done = s.t_empty + kAccBufs;
  s.tmem_slot = reinterpret_cast<uint32_t*>(s.mma_done + 1);
  s.abort_flag = s.tmem_slot + 1;
  s.epi_stop = s.tmem_slot + 2;
  return s;
}

// Column metadata for the epilogue: (scale, norm, local id, 0).  Columns past
// the leaf get norm = +inf so their distance is +inf and never selected.
__device__ __forceinline__ uint4 load_meta(const Params& p, uint64_t start, uint32_t cnt, uint32_t col) {
  if (col >= cnt) return make_uint4(0u, 0x7f800000u, 0xffffffffu, 0u);
  uint32_t lid = __ldg(p.members + start + col);
  if (lid >= p.resident_rows) {
    atomicOr(p.err_word, TESSA_DEVERR_BAD_ROW);
    return make_uint4(0u, 0x7f800000u, 0xffffffffu, 0u);
  }
  return make_uint4(__float_as_uint(__ldg(p.scales + lid)), __float_as_uint(__ldg(p.norms + lid)), lid, 0u);
}

// Selection set of one row: H unsorted slots in shared memory (slot-major so a
// warp's accesses are conflict-free), six blocks of six slots, block maxima
// (distance, slot) in registers; theta = max over the set.
struct RowSet {
  float bmax[kNBlk];
  uint32_t bslot[kNBlk];
  float theta;
  uint32_t gb;
  uint32_t fill;
};

__device__ __forceinline__ void set_rebuild(RowSet& rs, const float* sd, uint32_t row) {
#pragma unroll
  for (uint32_t b = 0; b < kNBlk; ++b) {
    float m = -INFINITY;
    uint32_t ms = b * kBlk;
#pragma unroll
    for (uint32_t t = 0; t < kBlk; ++t) {
      uint32_t sl = b * kBlk + t;
      float x = sd[sl * kBM + row];
      bool gt = x > m;
      m = gt ? x : m;
      ms = gt ? sl : ms;
    }
    rs.bmax[b] = m;
    rs.bslot[b] = ms;
  }
  rs.theta = rs.bmax[0];
  rs.gb = 0;
#pragma unroll
  for (uint32_t b = 1; b < kNBlk; ++b) {
    bool gt = rs.bmax[b] > rs.theta;
    rs.theta = gt ? rs.bmax[b] : rs.theta;
    rs.gb = gt ? b : rs.gb;
  }
}

// Insert (d, j) given d < theta (set full): overwrite the maximum, refresh
// its block and the global maximum.
__device__ __forceinline__ void set_replace_max(RowSet& rs, float* sd, uint16_t* sj, uint32_t row, float d,
                                                uint32_t j) {
  uint32_t slot = rs.bslot[0];
#pragma unroll
  for (uint32_t b = 1; b < kNBlk; ++b) slot = (rs.gb == b) ? rs.bslot[b] : slot;
  sd[slot * kBM + row] = d;
  sj[slot * kBM + row] = (uint16_t)j;
  uint32_t base = rs.gb * kBlk;
  float m = -INFINITY;
  uint32_t ms = base;
#pragma unroll
  for (uint32_t t = 0; t < kBlk; ++t) {
    float x = sd[(base + t) * kBM + row];
    bool gt = x > m;
    m = gt ? x : m;
    ms = gt ? base + t : ms;
  }
#pragma unroll
  for (uint32_t b = 0; b < kNBlk; ++b) {
    bool me = rs.gb == b;
    rs.bmax[b] = me ? m : rs.bmax[b];
    rs.bslot[b] = me ? ms : rs.bslot[b];
  }
  rs.theta = rs.bmax[0];
  rs.gb = 0;
#pragma unroll
  for (uint32_t b = 1; b < kNBlk; ++b) {
    bool gt = rs.bmax[b] > rs.theta;
    rs.theta = gt ? rs.bmax[b] : rs.theta;
    rs.gb = gt ? b : rs.gb;
  }
}

__device__ __forceinline__ uint32_t gid_of(const Params& p, uint64_t start, uint32_t j) {
  return __ldg(p.global_ids + __ldg(p.members + start + j));
}

// Finish one row: sort the set, verify order independence, write k results.
// Returns false if the row must be recomputed by the exact fallback.
__device__ bool finish_row(const Params& p, float* sd, uint16_t* sj, uint32_t row, uint32_t fill, bool complete,
                           uint64_t start, uint64_t out) {
  // Rank-sort the fill entries by (distance, position) back into the slots.
  float d[kSetSlots];
  uint32_t j[kSetSlots];
#pragma unroll
  for (uint32_t a = 0; a < kSetSlots; ++a) {
    bool live = a < fill;
    d[a] = live ? sd[a * kBM + row] : INFINITY;
    j[a] = live ? (uint32_t)sj[a * kBM + row] : 0x10000u + a;
  }
#pragma unroll
  for (uint32_t a = 0; a < kSetSlots; ++a) {
    uint32_t r = 0;
#pragma unroll
    for (uint32_t b = 0; b < kSetSlots; ++b) {
      bool lt = (d[b] < d[a]) | ((d[b] == d[a]) & (j[b] < j[a]));
      r += lt ? 1u : 0u;
    }
    if (a < fill) {
      sd[r * kBM + row] = d[a];
      sj[r * kBM + row] = (uint16_t)j[a];
    }
  }
  const uint32_t V = fill;
  const uint32_t k = p.k;
  uint32_t q = 0;  // output slots written
  uint32_t i = 0;
  while (q < k && i < V) {
    float di = sd[i * kBM + row];
    uint32_t e = i + 1;
    float prev = di;
    while (e < V) {
      float de = sd[e * kBM + row];
      if (!(fabsf(__fsub_rn(de, prev)) <= kTieEps)) break;
      prev = de;
      ++e;
    }
    uint32_t len = e - i;
    // The run holding rank k must end inside the set.
    if (q + len >= k && e == V && !complete) return false;
    if (len == 1) {
      p.out_ids[out + q] = gid_of(p, start, sj[i * kBM + row]);
      p.out_dists[out + q] = di;
      ++q;
    } else {
      // Tournament of the run under the eps/id rule: transitive iff the win
      // counts are 0..len-1 (then "<" orders the run by wins).
      if (len > 8) return false;
      float rd[8];
      uint32_t rg[8];
      for (uint32_t t = 0; t < len; ++t) {
        rd[t] = sd[(i + t) * kBM + row];
        rg[t] = gid_of(p, start, sj[(i + t) * kBM + row]);
      }
      uint32_t wins[8];
      uint32_t seen = 0;
      for (uint32_t t = 0; t < len; ++t) {
        uint32_t w = 0;
        for (uint32_t u = 0; u < len; ++u)
          if (u != t && stable_better(rd[t], rg[t], rd[u], rg[u])) ++w;
        wins[t] = w;
        seen |= 1u << w;
      }
      if (seen != (1u << len) - 1u) return false;
      for (uint32_t rank = 0; rank < len && q < k; ++rank) {
        uint32_t want = len - 1 - rank;
        for (uint32_t t = 0; t < len; ++t)
          if (wins[t] == want) {
            p.out_ids[out + q] = rg[t];
            p.out_dists[out + q] = rd[t];
          }
        ++q;
      }
    }
    i = e;
  }
  for (; q < k; ++q) {
    p.out_ids[out + q] = 0xffffffffu;
    p.out_dists[out + q] = 3.402823466e+38F;
  }
  return true;
}

__global__ void __launch_bounds__(kThreads, 1)
    leaf_topk_sq8_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                         const Params p) {
  extern __shared__ uint8_t smem_raw[];
  Smem s = carve(smem_raw, p.num_slabs, p.num_bstages);
  const uint32_t warp = threadIdx.x >> 5;
  const uint32_t lane = threadIdx.x & 31u;
  volatile uint32_t* abort_flag = s.abort_flag;

  if (threadIdx.x == 0) {
    mbar_init(s.a_full, 1);
    mbar_init(s.a_empty, 1);
    for (uint32_t i = 0; i < p.num_bstages; ++i) {
      mbar_init(&s.b_full[i], 1);
      mbar_init(&s.b_empty[i], 1);
    }
    for (uint32_t i = 0; i < kAccBufs; ++i) {
      mbar_init(&s.t_full[i], 1);
      mbar_init(&s.t_empty[i], kEpiThreads / 32);
    }
    mbar_init(s.mma_done, 1);
    *s.abort_flag = 0u;
    *s.epi_stop = 0u;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
  }
  if (warp == 1) {
    tmem_alloc(s.tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *s.tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t bstage = 0, bphase = 0, a_iter = 0;
      for (uint32_t tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++a_iter) {
        uint2 t = p.tiles[tile];
        uint64_t start = p.leaf_starts[t.x];
        uint32_t cnt = p.leaf_sizes[t.x];
        if (!mbar_wait(s.a_empty, (a_iter & 1u) ^ 1u, abort_flag, p.err_word, p.timeout_ns)) break;
        mbar_arrive_expect_tx(s.a_full, p.num_slabs * kASlabBytes);
        for (uint32_t sl = 0; sl < p.num_slabs; ++sl)
          tma_load_2d(&tmap_a, s.a + sl * kASlabBytes, s.a_full, (int32_t)(sl * kSlab), (int32_t)(start + t.y));
        uint32_t nchunks = (cnt + kBN - 1) / kBN;
        bool ok = true;
        for (uint32_t c = 0; c < nchunks && ok; ++c) {
          for (uint32_t sl = 0; sl < p.num_slabs; ++sl) {
            if (!mbar_wait(&s.b_empty[bstage], bphase ^ 1u, abort_flag, p.err_word, p.timeout_ns)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&s.b_full[bstage], kBStageBytes);
            tma_load_2d(&tmap_b, s.b + bstage * kBStageBytes, &s.b_full[bstage], (int32_t)(sl * kSlab),
                        (int32_t)(start + c * kBN));
            if (++bstage == p.num_bstages) {
              bstage = 0;
              bphase ^= 1u;
            }
          }
        }
        if (!ok) break;
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_i8(kBM, kBN);
      const uint32_t a_base = smem_u32(s.a);
      const uint32_t b_base = smem_u32(s.b);
      uint32_t bstage = 0, bphase = 0, acc = 0, a_iter = 0;
      bool ok = true;
      for (uint32_t tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x, ++a_iter) {
        uint2 t = p.tiles[tile];
        uint32_t cnt = p.leaf_sizes[t.x];
        if (!mbar_wait(s.a_full, a_iter & 1u, abort_flag, p.err_word, p.timeout_ns)) break;
        tc_fence_after();
        uint32_t nchunks = (cnt + kBN - 1) / kBN;
        for (uint32_t c = 0; c < nchunks && ok; ++c, ++acc) {
          uint32_t buf = acc % kAccBufs, use = acc / kAccBufs;
          if (!mbar_wait(&s.t_empty[buf], (use & 1u) ^ 1u, abort_flag, p.err_word, p.timeout_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          uint32_t tmem_d = tmem_base + buf * kBN;
          for (uint32_t sl = 0; sl < p.num_slabs; ++sl) {
            if (!mbar_wait(&s.b_full[bstage], bphase, abort_flag, p.err_word, p.timeout_ns)) {
              ok = false;
              break;
            }
            tc_fence_after();
            uint32_t a_addr = a_base + sl * kASlabBytes;
            uint32_t b_addr = b_base + bstage * kBStageBytes;
#pragma unroll
            for (uint32_t kk = 0; kk < kSlab / kMmaK; ++kk) {
              uint64_t ad = smem_desc_sw128(a_addr + kk * kMmaK);
              uint64_t bd = smem_desc_sw128(b_addr + kk * kMmaK);
              mma_i8_ss(tmem_d, ad, bd, idesc, (sl | kk) != 0u ? 1u : 0u);
            }
            mma_commit(&s.b_empty[bstage]);
            if (++bstage == p.num_bstages) {
              bstage = 0;
              bphase ^= 1u;
            }
          }
          if (ok) mma_commit(&s.t_full[buf]);
        }
        if (ok) mma_commit(s.a_empty);
      }
      // Every issued MMA must have landed before TMEM is released.
      mma_commit(s.mma_done);
      uint32_t dummy_abort = 0u;
      mbar_wait(s.mma_done, 0u, &dummy_abort, p.err_word, p.timeout_ns);
    }
  } else {
    // ------------------------------------------------------ epilogue
    const uint32_t ew = warp - 2;          // epilogue warp 0..3
    const uint32_t quad = warp & 3u;       // TMEM lane quadrant this warp may access
    const uint32_t et = threadIdx.x - 64;  // 0..127
    const uint32_t row_in_tile = quad * 32 + lane;
    float* stash = s.stash + ew * (kGroup * 32);
    uint32_t acc = 0;
    bool stop = false;
    for (uint32_t tile = blockIdx.x; tile < p.num_tiles && !stop; tile += gridDim.x) {
      uint2 t = p.tiles[tile];
      uint64_t start = p.leaf_starts[t.x];
      uint32_t cnt = p.leaf_sizes[t.x];
      uint32_t row = t.y + row_in_tile;
      bool valid = row < cnt;
      uint32_t lid_i = 0xfffffffeu;
      float s_i = 0.f, n_i = 0.f;
      if (valid) {
        lid_i = __ldg(p.members + start + row);
        if (lid_i >= p.resident_rows) {
          atomicOr(p.err_word, TESSA_DEVERR_BAD_ROW);
          valid = false;
          lid_i = 0xfffffffeu;
        } else {
          s_i = __ldg(p.scales + lid_i);
          n_i = __ldg(p.norms + lid_i);
        }
      }
      // Sentinel slots beyond H never become the maximum.
      for (uint32_t sl = p.h; sl < kSetSlots; ++sl) s.set_d[sl * kBM + row_in_tile] = -INFINITY;
      RowSet rs;
#pragma unroll
      for (uint32_t b = 0; b < kNBlk; ++b) {
        rs.bmax[b] = -INFINITY;
        rs.bslot[b] = b * kBlk;
      }
      rs.theta = valid ? INFINITY : -INFINITY;
      rs.gb = 0;
      rs.fill = 0;
      uint32_t offered = 0;  // candidates that went through the filter
      uint32_t nchunks = (cnt + kBN - 1) / kBN;
      s.meta[et] = load_meta(p, start, cnt, et);
      __syncwarp();
      named_bar_sync(1, kEpiThreads);
      for (uint32_t c = 0; c < nchunks; ++c, ++acc) {
        const uint4* meta = s.meta + (c & 1u) * kBN;
        uint4 nm = make_uint4(0, 0, 0, 0);
        if (c + 1 < nchunks) nm = load_meta(p, start, cnt, (c + 1) * kBN + et);
        uint32_t buf = acc % kAccBufs, use = acc / kAccBufs;
        bool ok = true;
        if (lane == 0) ok = mbar_wait(&s.t_full[buf], use & 1u, abort_flag, p.err_word, p.timeout_ns);
        ok = __shfl_sync(0xffffffffu, ok ? 1u : 0u, 0) != 0u;
        if (ok) {
          tc_fence_after();
#pragma unroll 1
          for (uint32_t g = 0; g < kGroups; ++g) {
            uint32_t v[32];
            tmem_ld_32x32b_x32(tmem_base + ((quad * 32u) << 16) + buf * kBN + g * kGroup, v);
            tmem_ld_wait();
            uint32_t mask = 0, real = 0;
            const float theta = rs.theta;
#pragma unroll
            for (uint32_t cc = 0; cc < kGroup; ++cc) {
              uint4 m = meta[g * kGroup + cc];
              float d = sq8_l2_from_dot((int)v[cc], s_i, n_i, __uint_as_float(m.x), __uint_as_float(m.y));
              bool cand = (m.z != lid_i) & (m.z != 0xffffffffu);
              real += cand ? 1u : 0u;
              bool pass = (d < theta) & cand;
              mask |= pass ? (1u << cc) : 0u;
              stash[cc * 32 + lane] = d;
            }
            offered += real;
            const uint32_t colbase = c * kBN + g * kGroup;
#pragma unroll 1
            while (mask) {
              uint32_t cc = __ffs(mask) - 1u;
              mask &= mask - 1u;
              float d = stash[cc * 32 + lane];
              if (d < rs.theta) {
                uint32_t j = colbase + cc;
                if (rs.fill < p.h) {
                  s.set_d[rs.fill * kBM + row_in_tile] = d;
                  s.set_j[rs.fill * kBM + row_in_tile] = (uint16_t)j;
                  ++rs.fill;
                  if (rs.fill == p.h) set_rebuild(rs, s.set_d, row_in_tile);
                } else {
                  set_replace_max(rs, s.set_d, s.set_j, row_in_tile, d, j);
                }
              }
            }
            __syncwarp();
          }
          tc_fence_before();
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.t_empty[buf]);
        if (c + 1 < nchunks) s.meta[((c + 1) & 1u) * kBN + et] = nm;
        __syncwarp();
        named_bar_sync(1, kEpiThreads);
        if (et == 0) *s.epi_stop = *abort_flag;
        named_bar_sync(1, kEpiThreads);
        if (*s.epi_stop) {
          stop = true;
          break;
        }
      }
      if (!stop && valid) {
        uint64_t out = (start + row) * (uint64_t)p.k;
        bool complete = offered <= rs.fill;  // the set holds every candidate of the row
        if (!finish_row(p, s.set_d, s.set_j, row_in_tile, rs.fill, complete, start, out)) {
          uint32_t slot = atomicAdd(p.fb_count, 1u);
          if (slot < p.fb_capacity)
            p.fb_list[slot] = make_uint2(t.x, row);
          else
            atomicOr(p.err_word, TESSA_DEVERR_BAD_TASK);
        }
      }
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// Exact fallback: recompute one listed row per warp with the reference's
// sequential insertion (ascending member position, CB:7229-7259).  Lane s holds
// list slot s; each candidate's rank is found with one ballot.
__global__ void __launch_bounds__(256) leaf_fallback_kernel(const int8_t* __restrict__ leaf_codes,
                                                             uint32_t padded_dim, const Params p) {
  extern __shared__ int4 fb_smem[];
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  const uint32_t words = padded_dim / 16u;  // int4 words per code row
  int4* rowbuf = fb_smem + warp * words;
  const uint32_t total = *p.fb_count;
  const uint32_t n = total < p.fb_capacity ? total : p.fb_capacity;
  const uint32_t k = p.k;
  for (uint32_t item = blockIdx.x * (blockDim.x >> 5) + warp; item < n; item += gridDim.x * (blockDim.x >> 5)) {
    uint2 e = p.fb_list[item];
    uint64_t start = p.leaf_starts[e.x];
    uint32_t cnt = p.leaf_sizes[e.x];
    uint32_t row = e.y;
    uint32_t lid_i = p.members[start + row];
    float s_i = p.scales[lid_i], n_i = p.norms[lid_i];
    const int4* rc = reinterpret_cast<const int4*>(leaf_codes + (start + row) * padded_dim);
    for (uint32_t w = lane; w < words; w += 32) rowbuf[w] = rc[w];
    __syncwarp();
    float bd = 3.402823466e+38F;
    uint32_t bi = 0xffffffffu;
    for (uint32_t c0 = 0; c0 < cnt; c0 += 32) {
      uint32_t jc = c0 + lane;
      float dj = INFINITY;
      uint32_t gj = 0xffffffffu, lj = 0xffffffffu;
      if (jc < cnt) {
        lj = p.members[start + jc];
        if (lj < p.resident_rows) {
          const int4* cc = reinterpret_cast<const int4*>(leaf_codes + (start + jc) * padded_dim);
          int dot = 0;
          for (uint32_t w = 0; w < words; ++w) {
            int4 x = rowbuf[w], y = cc[w];
            dot = __dp4a(x.x, y.x, dot);
            dot = __dp4a(x.y, y.y, dot);
            dot = __dp4a(x.z, y.z, dot);
            dot = __dp4a(x.w, y.w, dot);
          }
          dj = sq8_l2_from_dot(dot, s_i, n_i, p.scales[lj], p.norms[lj]);
          gj = p.global_ids[lj];
        } else {
          lj = lid_i;  // out-of-range ids were flagged by the main kernel; skip
        }
      }
      uint32_t lim = cnt - c0 < 32 ? cnt - c0 : 32;
      for (uint32_t t = 0; t < lim; ++t) {
        float d = __shfl_sync(0xffffffffu, dj, t);
        uint32_t g = __shfl_sync(0xffffffffu, gj, t);
        uint32_t l = __shfl_sync(0xffffffffu, lj, t);
        if (l == lid_i) continue;
        bool b = (lane < k) && stable_better(d, g, bd, bi);
        uint32_t m = __ballot_sync(0xffffffffu, b);
        if (!((m >> (k - 1)) & 1u)) continue;
        uint32_t live = k == 32 ? 0xffffffffu : ((1u << k) - 1u);
        uint32_t inv = ~m & live;
        uint32_t pos = inv ? (32u - __clz(inv)) : 0u;
        float ud = __shfl_up_sync(0xffffffffu, bd, 1);
        uint32_t ui = __shfl_up_sync(0xffffffffu, bi, 1);
        if (lane < k) {
          if (lane > pos) {
            bd = ud;
            bi = ui;
          } else if (lane == pos) {
            bd = d;
            bi = g;
          }
        }
      }
    }
    if (lane < k) {
      uint64_t out = (start + row) * (uint64_t)k + lane;
      p.out_ids[out] = bi;
      p.out_dists[out] = bd;
    }
    __syncwarp();
  }
}

// Gather code rows into leaf order: dst row p = src row members[p].
__global__ void gather_rows_kernel(const int8_t* __restrict__ src, const uint32_t* __restrict__ members,
                                   uint64_t rows, uint32_t row_bytes, int8_t* __restrict__ dst) {
  const uint32_t vec = row_bytes / 16u;
  for (uint64_t idx = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; idx < rows * vec;
       idx += (uint64_t)gridDim.x * blockDim.x) {
    uint64_t r = idx / vec;
    uint32_t v = (uint32_t)(idx - r * vec);
    const uint4* s = reinterpret_cast<const uint4*>(src + (uint64_t)members[r] * row_bytes) + v;
    reinterpret_cast<uint4*>(dst + r * row_bytes)[v] = *s;
  }
}

}  // namespace leaf

// ---------------------------------------------------------------- host side

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

// 2-D uint8 tensor map over `rows` x `row_bytes` (row stride = row_bytes), box
// of 128 bytes x box_rows, 128-byte swizzle, zero fill outside the tensor.
int make_code_tmap(CUtensorMap* map, const void* base, uint64_t rows, uint32_t row_bytes, uint32_t box_rows) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return -1;
  cuuint64_t dims[2] = {row_bytes, rows};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {leaf::kSlab, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -2;
}

int leaf_num_bstages(uint32_t padded_dim) {
  uint32_t slabs = (padded_dim + leaf::kSlab - 1) / leaf::kSlab;
  uint32_t fixed = leaf::smem_bytes(slabs, 0);
  if (fixed >= leaf::kSmemLimit) return 0;
  uint32_t st = (leaf::kSmemLimit - fixed) / leaf::kBStageBytes;
  if (st > leaf::kMaxBStages) st = leaf::kMaxBStages;
  return st >= 2 ? (int)st : 0;
}

// Returns 0, or a TESSA_ERR_* code.
int launch_leaf_topk_sq8(const LeafLaunch& L, cudaStream_t stream) {
  if (L.num_tiles == 0) return TESSA_OK;
  int nst = leaf_num_bstages(L.padded_dim);
  if (nst == 0) return TESSA_ERR_UNSUPPORTED;
  uint32_t slabs = (L.padded_dim + leaf::kSlab - 1) / leaf::kSlab;
  CUtensorMap ta, tb;
  if (make_code_tmap(&ta, L.leaf_codes, L.leaf_rows, L.padded_dim, leaf::kBM) != 0) return TESSA_ERR_CUDA;
  if (make_code_tmap(&tb, L.leaf_codes, L.leaf_rows, L.padded_dim, leaf::kBN) != 0) return TESSA_ERR_CUDA;
  leaf::Params prm;
  prm.scales = L.scales;
  prm.norms = L.norms;
  prm.global_ids = L.global_ids;
  prm.members = L.members;
  prm.leaf_starts = L.d_leaf_starts;
  prm.leaf_sizes = L.d_leaf_sizes;
  prm.tiles = L.d_tiles;
  prm.num_tiles = L.num_tiles;
  prm.num_slabs = slabs;
  prm.num_bstages = (uint32_t)nst;
  prm.k = L.k;
  prm.h = L.k + leaf::kExtra < leaf::kSetSlots ? L.k + leaf::kExtra : leaf::kSetSlots;
  prm.resident_rows = L.resident_rows;
  prm.out_ids = L.out_ids;
  prm.out_dists = L.out_dists;
  prm.err_word = L.d_err;
  prm.fb_count = L.d_fb_count;
  prm.fb_list = L.d_fb_list;
  prm.fb_capacity = L.fb_capacity;
  prm.timeout_ns = L.timeout_ns;
  uint32_t smem = leaf::smem_bytes(slabs, (uint32_t)nst);
  cudaError_t e = cudaFuncSetAttribute(leaf::leaf_topk_sq8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return TESSA_ERR_CUDA;
  e = cudaMemsetAsync(L.d_fb_count, 0, 4, stream);
  if (e != cudaSuccess) return TESSA_ERR_CUDA;
  uint32_t grid = L.num_tiles < (uint32_t)L.sm_count ? L.num_tiles : (uint32_t)L.sm_count;
  leaf::leaf_topk_sq8_kernel<<<grid, leaf::kThreads, smem, stream>>>(ta, tb, prm);
  if (cudaGetLastError() != cudaSuccess) return TESSA_ERR_CUDA;
  // Exact recomputation of the rows whose result depends on insertion order.
  uint32_t fb_smem = 8u * L.padded_dim;  // one code row per warp
  leaf::leaf_fallback_kernel<<<(unsigned)L.sm_count, 256, fb_smem, stream>>>(L.leaf_codes, L.padded_dim, prm);
  return cudaGetLastError() == cudaSuccess ? TESSA_OK : TESSA_ERR_CUDA;
}

int launch_gather_rows(const int8_t* src, const uint32_t* members, uint64_t rows, uint32_t row_bytes, int8_t* dst,
                       int sm_count, cudaStream_t stream) {
  if (rows == 0) return TESSA_OK;
  uint64_t work = rows * (row_bytes / 16u);
  uint64_t blocks = (work + 255) / 256;
  uint64_t cap = (uint64_t)sm_count * 8u;
  if (blocks > cap) blocks = cap;
  leaf::gather_rows_kernel<<<(unsigned)blocks, 256, 0, stream>>>(src, members, rows, row_bytes, dst);
  return cudaGetLastError() == cudaSuccess ? TESSA_OK : TESSA_ERR_CUDA;
}

}  // namespace tessa
