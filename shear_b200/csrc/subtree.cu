// Recursive TESSA leader partition of subtree tasks (the partition half of
// the reference's persistent kernel gpu_persistent_subtree_topk,
// shear-core/src/algorithm/pipnn/compute_backend.rs:16336-17381).
//
// B200 form: the reference runs one persistent kernel whose CTAs claim nodes
// from a device queue, one thread or one CTA per node, and scatters rows into
// children with atomics.  Here every level runs as a few wide launches over all
// queued nodes of all tasks (a round), driven by the host:
//   1. prepare_kernel   rows -> resident ids, leaders of every large node
//                       (evenly spaced positions, CB:12590-12601, or the span
//                       sampler of a retry, CB:5991-6017);
//   2. the tensor-core assignment kernel (assign_tc.cu) in slot mode: int8
//      dots on tcgen05 into TMEM, the reference's hash-tie insertion over
//      local_fanout slots with subtree-local tie ids (CB:6524-6578);
//   3. count_kernel     per (node, leader slot) row counts;
//   4. host decision    split / retry / balanced fallback per node (the EMIT
//                       phase, CB:15396-15505) and allocation of every child
//                       and leaf in node order;
//   5. scatter_kernel   stable scatter (rows keep ascending position; the rank
//                       of a row inside its child comes from per-chunk bitmaps
//                       and popcounts), leaves written as resident ids;
//   6. small_kernel     one CTA per subtree root of at most leaf_max rows that
//                       still splits (process_node, CB:12648-13048): hash
//                       bottom-k leaders, up to six attempts, child merging.
// Nothing here spins: every kernel is straight-line work over its node.
#include <algorithm>
#include <cmath>
#include <chrono>
#include <cstdio>
#include <cstring>
#include <new>
#include <vector>

#include "common.cuh"
#include "kernels.h"

namespace tessa {
namespace subtree {

constexpr uint32_t kSlots = 128;         // leaders per node (GPU_QUEUE_LEADER_STRIDE, CB:371)
constexpr uint32_t kSmallMaxRows = 2048; // small-path rows: n * fanout_second <= 4096, fanout_second >= 2
constexpr uint32_t kSmallMaxEntries = 4096;  // n * local_fanout (CB:12840 `running > 4096`)
constexpr uint32_t kTab = 1 + 2 * (kSlots + 1);  // small-node leaf table: count, (offset, size) pairs
constexpr uint64_t kLeafBit = 1ull << 63;    // scatter destination in the leaf arena

enum Mode : uint32_t { kSplit = 0, kBalanced = 1, kCopyNext = 2, kCopyLeaf = 3 };

struct NodeDesc {
  uint32_t off;      // arena position of the node's rows (subtree-local ids)
  uint32_t n;
  uint32_t task;
  uint32_t num;      // leaders
  uint32_t attempt;  // 0: evenly spaced leaders; > 0: span sampler of that attempt
  uint32_t lf;       // local fanout
  uint32_t depth;
  uint32_t mode;     // scatter mode
  uint64_t seed;
  uint64_t out;      // small path: leaf-arena reservation
};

__device__ __forceinline__ uint64_t hash64(uint64_t v) {
  v ^= v >> 30;
  v *= 0xbf58476d1ce4e5b9ull;
  v ^= v >> 27;
  v *= 0x94d049bb133111ebull;
  return v ^ (v >> 31);
}

__device__ __forceinline__ uint64_t tie_key(uint32_t point, uint32_t leader) {
  return hash64((((uint64_t)point) << 32) ^ (uint64_t)leader ^ 0x9e3779b97f4a7c15ull);
}

// Subtree roots: local ids 0..n-1.
__global__ void iota_kernel(const NodeDesc* nodes, uint32_t* cur) {
  const NodeDesc nd = nodes[blockIdx.x];
  for (uint32_t i = threadIdx.x; i < nd.n; i += blockDim.x) cur[nd.off + i] = i;
}

// Resident ids of a large node's rows and its leaders (local and resident).
__global__ void prepare_kernel(const NodeDesc* nodes, const uint32_t* cur, const uint32_t* task_members,
                               const uint64_t* task_off, uint32_t* member_res, uint32_t* leader_local,
                               uint32_t* leader_res) {
  const NodeDesc nd = nodes[blockIdx.x];
  const uint32_t* tm = task_members + task_off[nd.task];
  for (uint32_t i = threadIdx.x; i < nd.n; i += blockDim.x) member_res[nd.off + i] = tm[cur[nd.off + i]];
  for (uint32_t s = threadIdx.x; s < nd.num; s += blockDim.x) {
    uint32_t pos;
    if (nd.attempt == 0) {
      uint64_t o = ((uint64_t)s * nd.n) / nd.num;
      pos = (uint32_t)(o >= nd.n ? nd.n - 1u : o);
    } else {
      const uint32_t b = (uint32_t)(((uint64_t)s * nd.n) / nd.num);
      uint32_t e = (uint32_t)(((uint64_t)(s + 1u) * nd.n) / nd.num);
      if (e <= b) e = b + 1u;
      const uint64_t key = hash64(nd.seed ^ ((uint64_t)nd.attempt * 0xd6e8feb86659fd93ull) ^
                                  ((uint64_t)s * 0x9e3779b97f4a7c15ull));
      pos = b + (uint32_t)(key % (uint64_t)(e - b));
    }
    const uint32_t l = cur[nd.off + pos];
    leader_local[(uint64_t)blockIdx.x * kSlots + s] = l;
    leader_res[(uint64_t)blockIdx.x * kSlots + s] = tm[l];
  }
}

// Rows per leader slot of every large node.
__global__ void count_kernel(const NodeDesc* nodes, const uint32_t* slots, uint32_t* counts) {
  __shared__ uint32_t c[kSlots];
  const NodeDesc nd = nodes[blockIdx.x];
  for (uint32_t s = threadIdx.x; s < kSlots; s += blockDim.x) c[s] = 0;
  __syncthreads();
  const uint32_t* sl = slots + (uint64_t)nd.off * 4u;
  for (uint32_t i = threadIdx.x; i < nd.n; i += blockDim.x)
    for (uint32_t k = 0; k < nd.lf; ++k) {
      const uint32_t s = sl[(uint64_t)i * nd.lf + k];
      if (s < nd.num) atomicAdd(&c[s], 1u);
    }
  __syncthreads();
  for (uint32_t s = threadIdx.x; s < kSlots; s += blockDim.x) counts[(uint64_t)blockIdx.x * kSlots + s] = c[s];
}

__device__ __forceinline__ void put(uint64_t dest, uint32_t rank, uint32_t local, const uint32_t* tm,
                                    uint32_t* next, uint32_t* leaf_rows) {
  if (dest & kLeafBit)
    leaf_rows[(dest & ~kLeafBit) + rank] = tm[local];
  else
    next[dest + rank] = local;
}

// Scatter of one node's rows (block = 256 threads, one row per thread per
// chunk).  Split: a row's rank in child s is the number of earlier rows of the
// node assigned to s, from a per-chunk bitmap per slot plus the running count
// of the chunks before -- the sequential scatter order (ascending position).
// Assignment work items of large node j: (j, first row) for every 128 rows.
__global__ void work_kernel(const NodeDesc* nodes, const uint32_t* item_off, uint2* work) {
  const uint32_t j = blockIdx.x;
  const uint32_t n = nodes[j].n, base = item_off[j];
  for (uint32_t i = threadIdx.x; i * 128u < n; i += blockDim.x) work[base + i] = make_uint2(j, i * 128u);
}

__global__ void __launch_bounds__(256) scatter_kernel(const NodeDesc* nodes, const uint64_t* dests,
                                                      const uint32_t* cur, const uint32_t* slots,
                                                      const uint32_t* task_members, const uint64_t* task_off,
                                                      uint32_t* next, uint32_t* leaf_rows) {
  __shared__ uint32_t bits[kSlots][8];
  __shared__ uint32_t wpre[kSlots][8];
  __shared__ uint32_t tot[kSlots];
  __shared__ uint32_t running[kSlots];
  const NodeDesc nd = nodes[blockIdx.x];
  const uint64_t* dst = dests + nd.out;  // this node's destinations: 1, 2 or num entries
  const uint32_t* tm = task_members + task_off[nd.task];
  const uint32_t t = threadIdx.x;
  if (nd.mode != kSplit) {
    for (uint32_t i = t; i < nd.n; i += blockDim.x) {
      const uint32_t local = cur[nd.off + i];
      if (nd.mode == kBalanced)
        put(dst[i & 1u], i >> 1, local, tm, next, leaf_rows);
      else
        put(dst[0], i, local, tm, next, leaf_rows);
    }
    return;
  }
  for (uint32_t s = t; s < kSlots; s += blockDim.x) {
    running[s] = 0;
#pragma unroll
    for (uint32_t w = 0; w < 8; ++w) bits[s][w] = 0;
  }
  __syncthreads();
  const uint32_t* sl = slots + (uint64_t)nd.off * 4u;
  const uint32_t w = t >> 5, lanebit = 1u << (t & 31u), below = lanebit - 1u;
  for (uint32_t base = 0; base < nd.n; base += 256) {
    const uint32_t i = base + t;
    const bool valid = i < nd.n;
    uint32_t my[4] = {0xffffffffu, 0xffffffffu, 0xffffffffu, 0xffffffffu};
    uint32_t local = 0;
    if (valid) {
      local = cur[nd.off + i];
      for (uint32_t k = 0; k < nd.lf; ++k) {
        my[k] = sl[(uint64_t)i * nd.lf + k];
        if (my[k] < nd.num) atomicOr(&bits[my[k]][w], lanebit);
      }
    }
    __syncthreads();
    for (uint32_t s = t; s < nd.num; s += blockDim.x) {
      uint32_t run = 0;
#pragma unroll
      for (uint32_t ww = 0; ww < 8; ++ww) {
        wpre[s][ww] = run;
        run += __popc(bits[s][ww]);
      }
      tot[s] = run;
    }
    __syncthreads();
    if (valid)
      for (uint32_t k = 0; k < nd.lf; ++k) {
        const uint32_t s = my[k];
        if (s >= nd.num) continue;
        const uint32_t rank = running[s] + wpre[s][w] + __popc(bits[s][w] & below);
        put(dst[s], rank, local, tm, next, leaf_rows);
      }
    __syncthreads();
    for (uint32_t s = t; s < nd.num; s += blockDim.x) {
      running[s] += tot[s];
#pragma unroll
      for (uint32_t ww = 0; ww < 8; ++ww) bits[s][ww] = 0;
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------- small path

struct SmallParams {
  const NodeDesc* nodes;
  const uint32_t* cur;
  const uint32_t* task_members;
  const uint64_t* task_off;
  const int8_t* codes;
  const float* scales;
  const float* norms;
  uint32_t padded_dim;
  uint32_t leaf_max, leaf_min, max_leaders, fanout_second, root_depth;
  float psamp;
  uint32_t* leaf_rows;
  uint32_t* tables;  // kTab words per node
  uint32_t* err;
};

// CB:7044-7075
__host__ __device__ inline float adaptive_psamp(float base, uint32_t n, uint32_t depth) {
  float f = base;
  if (n >= 20000000u) f *= 0.05f;
  else if (n >= 10000000u) f *= 0.1f;
  else if (n >= 5000000u) f *= 0.2f;
  else if (n >= 1000000u) f *= 0.4f;
  else if (n >= 100000u) f *= 0.7f;
  if (depth > 4u) f *= 0.35f;
  else if (depth > 2u) f *= 0.5f;
  else if (depth > 0u) f *= 0.8f;
  if (f < 0.00005f) f = 0.00005f;
  if (f > 0.1f) f = 0.1f;
  return f;
}

// round(psamp * n) clamped to [2, max_leaders]; nvcc contracts the reference's
// `psamp_fraction * (float)n + 0.5f` (CB:12761, CB:12566) into one FMA.
__host__ __device__ inline uint32_t leader_count(float psamp, uint32_t n, uint32_t max_leaders) {
  uint32_t b = (uint32_t)fmaf(psamp, (float)n, 0.5f);
  if (b < 2u) b = 2u;
  if (b > max_leaders) b = max_leaders;
  return b;
}

// CB:7082-7101
__host__ __device__ inline bool meaningful_split(uint32_t parent, uint32_t max_child, uint32_t terminal) {
  if (parent <= terminal || max_child <= terminal) return true;
  if (max_child >= parent) return false;
  uint32_t m = parent >> 5;
  if (m < 32u) m = 32u;
  if (m >= parent) m = 1u;
  return max_child + m <= parent;
}

// CB:6524-6578 over n slots (as assign_tc.cu insertn)
__device__ void insert_slots(float d, uint32_t point, uint32_t leader, uint32_t slot, uint32_t n, float* bd,
                             uint32_t* bs, uint32_t* bl) {
  const uint32_t last = n - 1u;
  bool better = d < bd[last];
  uint64_t ck = 0;
  bool ready = false;
  if (fabsf(__fsub_rn(d, bd[last])) <= 2.0e-5f) {
    ck = tie_key(point, leader);
    ready = true;
    const uint64_t fk = tie_key(point, bl[last]);
    better = ck < fk || (ck == fk && leader < bl[last]);
  }
  if (!better) return;
  uint32_t pos = last;
  while (pos > 0) {
    bool before = d < bd[pos - 1];
    if (fabsf(__fsub_rn(d, bd[pos - 1])) <= 2.0e-5f) {
      if (!ready) {
        ck = tie_key(point, leader);
        ready = true;
      }
      const uint64_t pk = tie_key(point, bl[pos - 1]);
      before = ck < pk || (ck == pk && leader < bl[pos - 1]);
    }
    if (!before) break;
    bd[pos] = bd[pos - 1];
    bs[pos] = bs[pos - 1];
    bl[pos] = bl[pos - 1];
    --pos;
  }
  bd[pos] = d;
  bs[pos] = slot;
  bl[pos] = leader;
}

__device__ uint32_t merge_unique(const uint32_t* a, uint32_t na, const uint32_t* b, uint32_t nb, uint32_t* out) {
  uint32_t i = 0, j = 0, o = 0;
  while (i < na || j < nb) {
    uint32_t v;
    if (j >= nb || (i < na && a[i] <= b[j]))
      v = a[i++];
    else
      v = b[j++];
    if (o == 0 || out[o - 1] != v) out[o++] = v;
  }
  return o;
}

struct SmallSmem {
  uint32_t rows[kSmallMaxRows];
  uint32_t res[kSmallMaxRows];
  uint64_t keys[kSmallMaxRows];
  uint32_t slots[kSmallMaxEntries];
  uint32_t clustered[kSmallMaxEntries];
  uint32_t merged[kSmallMaxEntries];
  uint32_t small[kSmallMaxEntries];
  uint32_t tmp[kSmallMaxEntries];
  uint32_t leaders[kSlots], lres[kSlots], counts[kSlots], starts[kSlots], writes[kSlots];
  uint32_t child_off[kSlots + 1], child_cnt[kSlots + 1];
  uint32_t nchild, ok, num, lf, merged_rows, whole;
};

// process_node (CB:12648-13048) for one subtree root of at most leaf_max rows
// that splits (root fanout probe).  Children here are never above the node
// size, so every child is a leaf; they are written as resident ids into the
// node's reservation and listed in its table.
__global__ void __launch_bounds__(256) small_kernel(const SmallParams p) {
  extern __shared__ uint8_t smem_raw[];
  SmallSmem& S = *reinterpret_cast<SmallSmem*>(smem_raw);
  const NodeDesc nd = p.nodes[blockIdx.x];
  const uint32_t t = threadIdx.x, n = nd.n;
  const uint32_t* tm = p.task_members + p.task_off[nd.task];
  for (uint32_t i = t; i < n; i += blockDim.x) {
    S.rows[i] = p.cur[nd.off + i];
    S.res[i] = tm[S.rows[i]];
  }
  const uint32_t rd = nd.depth >= p.root_depth ? nd.depth - p.root_depth : 0u;
  uint32_t max_leaders = p.max_leaders < n ? p.max_leaders : n;
  if (max_leaders < 2u) max_leaders = 2u;
  const uint32_t base = leader_count(adaptive_psamp(p.psamp, n, nd.depth), n, max_leaders);
  uint32_t requested = rd == 0u ? p.fanout_second : 1u;
  if (requested < 1u) requested = 1u;
  if (t == 0) {
    S.ok = 0;
    S.whole = 0;
  }
  __syncthreads();
  const uint32_t pd = p.padded_dim;
  for (uint32_t attempt = 0; attempt < 6u; ++attempt) {
    uint32_t num = base << attempt;
    if (num > max_leaders) num = max_leaders;
    const uint32_t lf = requested < num ? requested : num;
    // hash bottom-num leaders in (key, point) order
    for (uint32_t i = t; i < n; i += blockDim.x)
      S.keys[i] = hash64(nd.seed ^ ((uint64_t)attempt * 0xbf58476d1ce4e5b9ull) ^ (((uint64_t)nd.depth) << 19) ^
                         (((uint64_t)i) << 7) ^ (((uint64_t)S.rows[i]) << 31));
    __syncthreads();
    for (uint32_t i = t; i < n; i += blockDim.x) {
      const uint64_t ki = S.keys[i];
      const uint32_t pi = S.rows[i];
      uint32_t rank = 0;
      for (uint32_t j = 0; j < n; ++j) {
        const uint64_t kj = S.keys[j];
        rank += (kj < ki || (kj == ki && S.rows[j] < pi)) ? 1u : 0u;
      }
      if (rank < num) {
        S.leaders[rank] = pi;
        S.lres[rank] = S.res[i];
      }
    }
    __syncthreads();
    // assignment: best lf slots per row (int8 dots, contracted distance)
    for (uint32_t i = t; i < n; i += blockDim.x) {
      const int4* rc = reinterpret_cast<const int4*>(p.codes + (uint64_t)S.res[i] * pd);
      const float np = p.norms[S.res[i]], sp = p.scales[S.res[i]];
      float bd[4] = {3.402823466e+38F, 3.402823466e+38F, 3.402823466e+38F, 3.402823466e+38F};
      uint32_t bs[4] = {0xffffffffu, 0xffffffffu, 0xffffffffu, 0xffffffffu};
      uint32_t bl[4] = {0xffffffffu, 0xffffffffu, 0xffffffffu, 0xffffffffu};
      for (uint32_t s = 0; s < num; ++s) {
        const uint32_t lr = S.lres[s];
        const int4* lc = reinterpret_cast<const int4*>(p.codes + (uint64_t)lr * pd);
        int dot = 0;
        for (uint32_t q = 0; q < pd / 16u; ++q) {
          const int4 a = rc[q], b = lc[q];
          dot = __dp4a(a.x, b.x, dot);
          dot = __dp4a(a.y, b.y, dot);
          dot = __dp4a(a.z, b.z, dot);
          dot = __dp4a(a.w, b.w, dot);
        }
        const float nn = __fadd_rn(np, p.norms[lr]);
        const float tt = __fmul_rn(__fmul_rn(2.0f, sp), p.scales[lr]);
        float d = __fmaf_rn(-tt, __int2float_rn(dot), nn);
        if (d <= 0.0f) d = 0.0f;
        insert_slots(d, S.rows[i], S.leaders[s], s, lf, bd, bs, bl);
      }
      for (uint32_t k = 0; k < lf; ++k) S.slots[i * lf + k] = bs[k];
    }
    __syncthreads();
    if (t == 0) {
      // clustering and child formation (CB:12815-12914), sequential
      for (uint32_t s = 0; s < num; ++s) S.counts[s] = 0;
      bool bad = false;
      for (uint32_t i = 0; i < n * lf; ++i) {
        if (S.slots[i] >= num) bad = true;
        else S.counts[S.slots[i]]++;
      }
      uint32_t running = 0;
      for (uint32_t s = 0; s < num; ++s) {
        S.starts[s] = running;
        S.writes[s] = running;
        running += S.counts[s];
      }
      if (running > kSmallMaxEntries) bad = true;
      if (bad) atomicOr(p.err, TESSA_DEVERR_BAD_TASK);
      for (uint32_t i = 0; i < n && !bad; ++i)
        for (uint32_t k = 0; k < lf; ++k) S.clustered[S.writes[S.slots[i * lf + k]]++] = S.rows[i];
      uint32_t nchild = 0, merged_rows = 0, small_len = 0, max_child = 0;
      for (uint32_t s = 0; s < num && !bad; ++s) {
        const uint32_t cnt = S.counts[s];
        if (cnt == 0) continue;
        const uint32_t* seg = S.clustered + S.starts[s];
        if (cnt < p.leaf_min) {
          const uint32_t m = merge_unique(S.small, small_len, seg, cnt, S.tmp);
          for (uint32_t i = 0; i < m; ++i) S.small[i] = S.tmp[i];
          small_len = m;
          if (small_len >= p.leaf_min) {
            for (uint32_t i = 0; i < small_len; ++i) S.merged[merged_rows + i] = S.small[i];
            S.child_off[nchild] = merged_rows;
            S.child_cnt[nchild] = small_len;
            merged_rows += small_len;
            if (small_len > max_child) max_child = small_len;
            nchild++;
            small_len = 0;
          }
        } else {
          S.child_off[nchild] = merged_rows;
          S.child_cnt[nchild] = cnt;
          for (uint32_t i = 0; i < cnt; ++i) S.merged[merged_rows + i] = seg[i];
          merged_rows += cnt;
          if (cnt > max_child) max_child = cnt;
          nchild++;
        }
      }
      if (small_len > 0 && nchild > 0) {
        const uint32_t last = nchild - 1;
        if (S.child_cnt[last] + small_len <= p.leaf_max) {
          const uint32_t m = merge_unique(S.merged + S.child_off[last], S.child_cnt[last], S.small, small_len, S.tmp);
          for (uint32_t i = 0; i < m; ++i) S.merged[S.child_off[last] + i] = S.tmp[i];
          merged_rows = S.child_off[last] + m;
          S.child_cnt[last] = m;
          if (m > max_child) max_child = m;
          small_len = 0;
        }
      }
      if (small_len > 0) {
        for (uint32_t i = 0; i < small_len; ++i) S.merged[merged_rows + i] = S.small[i];
        S.child_off[nchild] = merged_rows;
        S.child_cnt[nchild] = small_len;
        merged_rows += small_len;
        if (small_len > max_child) max_child = small_len;
        nchild++;
      }
      S.nchild = nchild;
      S.merged_rows = merged_rows;
      S.ok = (!bad && nchild > 1 && meaningful_split(n, max_child, p.leaf_max)) ? 1u : 0u;
      if (bad) S.whole = 2;  // stop: error already flagged
    }
    __syncthreads();
    if (S.ok || S.whole == 2 || num >= max_leaders) break;
  }
  uint32_t* tab = p.tables + (uint64_t)blockIdx.x * kTab;
  uint32_t* out = p.leaf_rows + nd.out;
  if (S.whole == 2) {
    if (t == 0) tab[0] = 0;
    return;
  }
  if (!S.ok) {
    // no split: the node itself is one leaf (n <= leaf_max here)
    for (uint32_t i = t; i < n; i += blockDim.x) out[i] = S.res[i];
    if (t == 0) {
      tab[0] = 1;
      tab[1] = 0;
      tab[2] = n;
    }
    return;
  }
  for (uint32_t i = t; i < S.merged_rows; i += blockDim.x) out[i] = tm[S.merged[i]];
  if (t == 0) {
    tab[0] = S.nchild;
    for (uint32_t c = 0; c < S.nchild; ++c) {
      tab[1 + 2 * c] = S.child_off[c];
      tab[2 + 2 * c] = S.child_cnt[c];
      if (S.child_cnt[c] > p.leaf_max) atomicOr(p.err, TESSA_DEVERR_BAD_TASK);
    }
  }
}

// ------------------------------------------------------------- host driver

struct Buf {
  void* ptr = nullptr;
  size_t bytes = 0;
  bool ensure(size_t need) {
    if (need <= bytes) return true;
    if (ptr) cudaFree(ptr);
    ptr = nullptr;
    bytes = 0;
    if (cudaMalloc(&ptr, need ? need : 16) != cudaSuccess) {
      ptr = nullptr;
      return false;
    }
    bytes = need ? need : 16;
    return true;
  }
  void release() {
    if (ptr) cudaFree(ptr);
    ptr = nullptr;
    bytes = 0;
  }
  template <class T>
  T* as() const {
    return reinterpret_cast<T*>(ptr);
  }
};

}  // namespace subtree

// Pinned host memory for one phase's copies: the host tables of a phase are
// packed here and copied with cudaMemcpyAsync from pinned memory (no driver
// staging of pageable memory, no host-side wait).  A stage is refilled only
// after the stream has passed the copies that read it (the round's syncs).
struct PinnedStage {
  uint8_t* p = nullptr;
  size_t cap = 0;
  std::vector<uint8_t> host;  // bytes collected for the next flush
  struct Item {
    void* dst;
    size_t off, bytes;
  };
  std::vector<Item> items;
  void add(void* dst, const void* src, size_t bytes) {
    const size_t off = (host.size() + 15) & ~size_t(15);
    host.resize(off + bytes);
    if (bytes) memcpy(host.data() + off, src, bytes);
    items.push_back(Item{dst, off, bytes});
  }
  // copies every item to its device destination on `st`
  cudaError_t flush(cudaStream_t st) {
    if (host.size() > cap) {
      cudaError_t e = cudaStreamSynchronize(st);
      if (e != cudaSuccess) return e;
      if (p) cudaFreeHost(p);
      p = nullptr;
      cap = 0;
      const size_t want = host.size() + host.size() / 4 + 4096;
      e = cudaHostAlloc(reinterpret_cast<void**>(&p), want, cudaHostAllocDefault);
      if (e != cudaSuccess) return e;
      cap = want;
    }
    if (!host.empty()) memcpy(p, host.data(), host.size());
    for (const Item& it : items) {
      if (!it.bytes) continue;
      const cudaError_t e = cudaMemcpyAsync(it.dst, p + it.off, it.bytes, cudaMemcpyHostToDevice, st);
      if (e != cudaSuccess) return e;
    }
    host.clear();
    items.clear();
    return cudaSuccess;
  }
  void release() {
    if (p) cudaFreeHost(p);
    p = nullptr;
    cap = 0;
  }
};

struct PinnedBuf {
  void* p = nullptr;
  size_t cap = 0;
  bool ensure(size_t need) {
    if (need <= cap) return true;
    if (p) cudaFreeHost(p);
    p = nullptr;
    cap = 0;
    if (cudaHostAlloc(&p, need + need / 4 + 64, cudaHostAllocDefault) != cudaSuccess) {
      p = nullptr;
      return false;
    }
    cap = need + need / 4 + 64;
    return true;
  }
  void release() {
    if (p) cudaFreeHost(p);
    p = nullptr;
    cap = 0;
  }
  template <class T>
  T* as() const {
    return reinterpret_cast<T*>(p);
  }
};

struct SubtreeState {
  subtree::Buf cur, next, member_res, slots, leader_local, leader_res, counts, dests, nodes, small_nodes, tables,
      task_off, t_moff, t_mcnt, t_loff, t_lcnt, t_rh, t_out, work, item_off;
  // phase boundaries of a round: assignment, scatter, small path
  cudaEvent_t ev[6] = {nullptr, nullptr, nullptr, nullptr, nullptr, nullptr};
  // leaf-ordered code copies run on a side stream after each round's scatter
  cudaStream_t side = nullptr;
  cudaEvent_t round_done = nullptr, side_done = nullptr;
  bool side_stream() {
    if (!side && cudaStreamCreateWithFlags(&side, cudaStreamNonBlocking) != cudaSuccess) return false;
    if (!round_done && cudaEventCreateWithFlags(&round_done, cudaEventDisableTiming) != cudaSuccess) return false;
    if (!side_done && cudaEventCreateWithFlags(&side_done, cudaEventDisableTiming) != cudaSuccess) return false;
    return true;
  }
  // pinned staging: per-phase host tables, counts and small-node tables back
  PinnedStage stage_assign, stage_scatter, stage_small;
  PinnedBuf h_counts, h_tables, h_bits;
  bool events() {
    for (auto& e : ev)
      if (!e && cudaEventCreate(&e) != cudaSuccess) return false;
    return true;
  }
  void release() {
    subtree::Buf* all[] = {&cur, &next, &member_res, &slots, &leader_local, &leader_res, &counts, &dests, &nodes,
                           &small_nodes, &tables, &task_off, &t_moff, &t_mcnt, &t_loff, &t_lcnt, &t_rh, &t_out,
                           &work, &item_off};
    for (auto* b : all) b->release();
    stage_assign.release();
    stage_scatter.release();
    stage_small.release();
    h_counts.release();
    h_tables.release();
    h_bits.release();
  }
};

SubtreeState* subtree_state_new() { return new (std::nothrow) SubtreeState(); }
void subtree_state_free(SubtreeState* s) {
  if (!s) return;
  s->release();
  for (auto& e : s->ev)
    if (e) cudaEventDestroy(e);
  if (s->side) {
    cudaStreamSynchronize(s->side);
    cudaStreamDestroy(s->side);
  }
  if (s->round_done) cudaEventDestroy(s->round_done);
  if (s->side_done) cudaEventDestroy(s->side_done);
  delete s;
}

namespace {

using subtree::NodeDesc;

struct HNode {
  uint32_t task, off, n, depth, attempt, num, lf;
  uint64_t seed;
};

#define ST_CUDA(expr)                                                                         \
  do {                                                                                        \
    cudaError_t _e = (expr);                                                                  \
    if (_e != cudaSuccess) {                                                                  \
      char _m[256];                                                                           \
      snprintf(_m, sizeof _m, "%s: %s", #expr, cudaGetErrorString(_e));                       \
      return set_last_error(_e == cudaErrorMemoryAllocation ? TESSA_ERR_OOM : TESSA_ERR_CUDA, _m); \
    }                                                                                         \
  } while (0)

#define ST_ALLOC(buf, bytes)                                                               \
  do {                                                                                     \
    if (!(buf).ensure(bytes)) return set_last_error(TESSA_ERR_OOM, "subtree scratch allocation failed"); \
  } while (0)

uint64_t child_seed(uint64_t seed, uint32_t child, uint32_t len) {
  return seed ^ ((uint64_t)child * 0x94d049bb133111ebull) ^ (((uint64_t)len) << 23);
}

enum Kind { kLeafNode, kSmall, kLarge };

}  // namespace

int subtree_partition(SubtreeState* S, const tessa_subtree_args& a, SubtreeStats* stats, uint32_t* d_err, int sm_count,
                      uint64_t timeout_ns, cudaStream_t st) {
  using namespace subtree;
  const uint32_t fs = a.fanout_second < 1u ? 1u : a.fanout_second;
  // every task row lands in at most fanout_second arena rows: the scratch is
  // sized by the tasks' rows, not by the whole member array they index
  uint64_t task_rows = 0;
  for (uint32_t t = 0; t < a.task_count; ++t) task_rows += a.task_counts[t];
  const uint64_t arena_cap = (uint64_t)fs * task_rows + 16;
  const uint32_t max_leaders = a.max_leaders < kSlots ? a.max_leaders : kSlots;
  ST_ALLOC(S->cur, arena_cap * 4);
  ST_ALLOC(S->next, arena_cap * 4);
  ST_ALLOC(S->member_res, arena_cap * 4);
  ST_ALLOC(S->slots, arena_cap * 16);
  ST_ALLOC(S->task_off, (size_t)a.task_count * 8 + 8);
  if (a.task_count) ST_CUDA(cudaMemcpyAsync(S->task_off.ptr, a.task_offsets, (size_t)a.task_count * 8,
                                            cudaMemcpyHostToDevice, st));
  // arena rows that end up in no leaf (the unused part of a small node's
  // reservation) read as 0xffffffff, never as stale ids
  if (a.leaf_rows_capacity) ST_CUDA(cudaMemsetAsync(a.leaf_rows, 0xff, (size_t)a.leaf_rows_capacity * 4, st));
  *stats = SubtreeStats{};
  const auto wall0 = std::chrono::steady_clock::now();
  if (!S->events()) return set_last_error(TESSA_ERR_CUDA, "subtree timing events could not be created");
  using clk = std::chrono::steady_clock;
  auto ms_since = [](clk::time_point t0) {
    return std::chrono::duration<float, std::milli>(clk::now() - t0).count();
  };
  auto elapsed = [&](int a0, int a1) {
    float ms = 0.f;
    return cudaEventElapsedTime(&ms, S->ev[a0], S->ev[a1]) == cudaSuccess ? ms : 0.f;
  };

  // round 0: one root node per non-empty task, rows 0..n-1
  std::vector<HNode> nodes;
  uint64_t cur_len = 0;
  for (uint32_t t = 0; t < a.task_count; ++t) {
    if (a.task_counts[t] == 0) continue;
    nodes.push_back(HNode{t, (uint32_t)cur_len, a.task_counts[t], a.root_depth, 0u, 0u, 0u, a.task_seeds[t]});
    cur_len += a.task_counts[t];
  }
  if (cur_len >= 0xffffffffull) return set_last_error(TESSA_ERR_UNSUPPORTED, "subtree rows beyond 2^32");
  {
    std::vector<NodeDesc> d(nodes.size());
    for (size_t i = 0; i < nodes.size(); ++i) d[i] = NodeDesc{nodes[i].off, nodes[i].n, nodes[i].task, 0, 0, 0, 0, 0, 0, 0};
    ST_ALLOC(S->nodes, d.size() * sizeof(NodeDesc) + 16);
    if (!d.empty()) {
      ST_CUDA(cudaMemcpyAsync(S->nodes.ptr, d.data(), d.size() * sizeof(NodeDesc), cudaMemcpyHostToDevice, st));
      iota_kernel<<<(unsigned)d.size(), 256, 0, st>>>(S->nodes.as<NodeDesc>(), S->cur.as<uint32_t>());
      ST_CUDA(cudaGetLastError());
      stats->launches++;
    }
  }

  struct LeafEnt {
    uint64_t start;
    uint32_t size, task;
  };
  std::vector<LeafEnt> leaves;
  uint64_t leaf_used = 0;
  auto leaf_alloc = [&](uint64_t n, uint64_t* at) -> bool {
    if (leaf_used + n > a.leaf_rows_capacity) return false;
    *at = leaf_used;
    leaf_used += n;
    return true;
  };

  const uint32_t small_smem = (uint32_t)sizeof(SmallSmem);
  ST_CUDA(cudaFuncSetAttribute(small_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)small_smem));

  if (a.leaf_codes && !S->side_stream())
    return set_last_error(TESSA_ERR_CUDA, "subtree side stream could not be created");
  // on every way out (errors included) the caller's stream follows the copies
  struct SideJoin {
    SubtreeState* S;
    cudaStream_t st;
    bool on;
    ~SideJoin() {
      if (on && cudaEventRecord(S->side_done, S->side) == cudaSuccess) cudaStreamWaitEvent(st, S->side_done, 0);
    }
  } side_join{S, st, a.leaf_codes != nullptr};
  while (!nodes.empty()) {
    stats->rounds++;
    const uint64_t leaf_round0 = leaf_used;
    auto t_prep = clk::now();
    // ---- classify
    std::vector<Kind> kind(nodes.size());
    std::vector<uint32_t> large_idx, small_idx;
    for (size_t q = 0; q < nodes.size(); ++q) {
      HNode& nd = nodes[q];
      const uint32_t rd = nd.depth >= a.root_depth ? nd.depth - a.root_depth : 0u;
      const bool probe = rd == 0u && fs > 1u && nd.n > 1u;
      const bool probe_over = probe && (uint64_t)nd.n * fs > a.small_node_limit;
      if (nd.n <= a.leaf_max && !probe_over) {
        if (!probe) {
          kind[q] = kLeafNode;
          continue;
        }
        if (nd.depth >= a.max_depth)
          return set_last_error(TESSA_ERR_PARTITION, "subtree node at max_depth cannot split");
        kind[q] = kSmall;
        small_idx.push_back((uint32_t)q);
        continue;
      }
      if (nd.depth >= a.max_depth)
        return set_last_error(TESSA_ERR_PARTITION, "subtree node above leaf_max at max_depth (oversized terminal)");
      kind[q] = kLarge;
      if (nd.attempt == 0) {
        uint32_t retry_max = nd.n < 2u ? 2u : nd.n;
        if (retry_max > kSlots) retry_max = kSlots;
        uint32_t ml = max_leaders < retry_max ? max_leaders : retry_max;
        if (ml < 2u) ml = 2u;
        const uint32_t base = leader_count(adaptive_psamp(a.psamp_fraction, nd.n, nd.depth), nd.n, ml);
        const uint32_t requested = rd == 0u ? fs : 1u;
        nd.num = base;
        nd.lf = requested < base ? requested : base;
      }
      large_idx.push_back((uint32_t)q);
    }

    // ---- large nodes: leaders, assignment, counts
    std::vector<uint32_t> counts(large_idx.size() * kSlots);
    if (!large_idx.empty()) {
      const size_t L = large_idx.size();
      std::vector<NodeDesc> d(L);
      std::vector<uint32_t> moff(L), mcnt(L), loff(L), lcnt(L), rh(L);
      std::vector<uint64_t> tout(L);
      // work items (node, first row) are written on the device from each
      // node's first item index
      std::vector<uint32_t> item_off(L + 1);
      uint64_t items = 0;
      uint32_t nb_max = 0;
      for (size_t j = 0; j < L; ++j) {
        const HNode& nd = nodes[large_idx[j]];
        d[j] = NodeDesc{nd.off, nd.n, nd.task, nd.num, nd.attempt, nd.lf, nd.depth, 0u, nd.seed, 0};
        moff[j] = nd.off;
        mcnt[j] = nd.n;
        loff[j] = (uint32_t)(j * kSlots);
        lcnt[j] = nd.num;
        rh[j] = nd.lf;
        tout[j] = (uint64_t)nd.off * 4u;
        nb_max = std::max(nb_max, nd.num);
        item_off[j] = (uint32_t)items;
        items += (nd.n + 127u) / 128u;
      }
      if (L * kSlots >= 0xffffffffull) return set_last_error(TESSA_ERR_UNSUPPORTED, "too many subtree nodes");
      ST_ALLOC(S->nodes, L * sizeof(NodeDesc));
      ST_ALLOC(S->leader_local, L * kSlots * 4);
      ST_ALLOC(S->leader_res, L * kSlots * 4);
      ST_ALLOC(S->counts, L * kSlots * 4);
      ST_ALLOC(S->t_moff, L * 4);
      ST_ALLOC(S->t_mcnt, L * 4);
      ST_ALLOC(S->t_loff, L * 4);
      ST_ALLOC(S->t_lcnt, L * 4);
      ST_ALLOC(S->t_rh, L * 4);
      ST_ALLOC(S->t_out, L * 8);
      if (items >= 0xffffffffull) return set_last_error(TESSA_ERR_UNSUPPORTED, "too many subtree work items");
      item_off[L] = (uint32_t)items;
      ST_ALLOC(S->work, items * 8);
      ST_ALLOC(S->item_off, (L + 1) * 4);
      {
        PinnedStage& g = S->stage_assign;
        g.add(S->nodes.ptr, d.data(), L * sizeof(NodeDesc));
        g.add(S->t_moff.ptr, moff.data(), L * 4);
        g.add(S->t_mcnt.ptr, mcnt.data(), L * 4);
        g.add(S->t_loff.ptr, loff.data(), L * 4);
        g.add(S->t_lcnt.ptr, lcnt.data(), L * 4);
        g.add(S->t_rh.ptr, rh.data(), L * 4);
        g.add(S->t_out.ptr, tout.data(), L * 8);
        g.add(S->item_off.ptr, item_off.data(), (L + 1) * 4);
        ST_CUDA(g.flush(st));
      }
      stats->host_prep_ms += ms_since(t_prep);
      ST_CUDA(cudaEventRecord(S->ev[0], st));
      work_kernel<<<(unsigned)L, 128, 0, st>>>(S->nodes.as<NodeDesc>(), S->item_off.as<uint32_t>(),
                                               S->work.as<uint2>());
      prepare_kernel<<<(unsigned)L, 256, 0, st>>>(S->nodes.as<NodeDesc>(), S->cur.as<uint32_t>(), a.task_members,
                                                  S->task_off.as<uint64_t>(), S->member_res.as<uint32_t>(),
                                                  S->leader_local.as<uint32_t>(), S->leader_res.as<uint32_t>());
      ST_CUDA(cudaGetLastError());
      assign::Params prm{};
      prm.codes = a.codes;
      prm.scales = a.scales;
      prm.sq8_norms = a.sq8_norms;
      prm.global_ids = nullptr;
      prm.resident_rows = a.resident_rows;
      prm.padded_dim = a.padded_dim;
      prm.members = S->member_res.as<uint32_t>();
      prm.leaders = S->leader_res.as<uint32_t>();
      prm.t_moff = S->t_moff.as<uint32_t>();
      prm.t_mcnt = S->t_mcnt.as<uint32_t>();
      prm.t_loff = S->t_loff.as<uint32_t>();
      prm.t_lcnt = S->t_lcnt.as<uint32_t>();
      prm.t_rh = S->t_rh.as<uint32_t>();
      prm.t_out = S->t_out.as<uint64_t>();
      prm.work = S->work.as<uint2>();
      prm.num_work = (uint32_t)items;
      prm.fused = 1;
      prm.out_ids = nullptr;
      prm.out_dists = nullptr;
      prm.err_word = d_err;
      prm.timeout_ns = timeout_ns;
      prm.member_tie = S->cur.as<uint32_t>();
      prm.leader_tie = S->leader_local.as<uint32_t>();
      prm.out_slots = S->slots.as<uint32_t>();
      int rc = launch_assign_sq8_tc(prm, nb_max, sm_count, st);
      if (rc != TESSA_OK) return set_last_error(rc, "subtree assignment launch failed");
      stats->launches += 4;  // work items, prepare, assignment, count
      count_kernel<<<(unsigned)L, 256, 0, st>>>(S->nodes.as<NodeDesc>(), S->slots.as<uint32_t>(),
                                                S->counts.as<uint32_t>());
      ST_CUDA(cudaGetLastError());
      ST_CUDA(cudaEventRecord(S->ev[1], st));
      if (!S->h_counts.ensure(L * kSlots * 4) || !S->h_bits.ensure(8))
        return set_last_error(TESSA_ERR_OOM, "subtree pinned staging allocation failed");
      ST_CUDA(cudaMemcpyAsync(S->h_counts.p, S->counts.ptr, L * kSlots * 4, cudaMemcpyDeviceToHost, st));
      ST_CUDA(cudaMemcpyAsync(S->h_bits.p, d_err, 4, cudaMemcpyDeviceToHost, st));
      const auto t_wait = clk::now();
      ST_CUDA(cudaStreamSynchronize(st));
      stats->sync_wait_ms += ms_since(t_wait);
      const uint32_t bits = *S->h_bits.as<uint32_t>();
      memcpy(counts.data(), S->h_counts.p, L * kSlots * 4);
      if (bits) return bits & TESSA_DEVERR_TIMEOUT ? set_last_error(TESSA_ERR_TIMEOUT, "subtree assignment timed out")
                                                   : set_last_error(TESSA_ERR_BAD_TASK, "subtree assignment failed");
      stats->large_assignments += (uint32_t)L;
      stats->assign_ms += elapsed(0, 1);
    }

    // ---- decisions and allocation in node order
    const auto t_decide = clk::now();
    std::vector<HNode> next_nodes;
    uint64_t next_len = 0;
    // scatter plan for leaf-all and large nodes
    std::vector<NodeDesc> sc;
    std::vector<uint64_t> dests;
    sc.reserve(nodes.size());
    dests.reserve(nodes.size() * 8);
    // small nodes: reservation and position in the leaf list
    std::vector<NodeDesc> sm;
    std::vector<size_t> sm_leaf_pos;
    size_t li = 0;
    auto push_next = [&](const HNode& proto, uint32_t n, uint64_t* dest) -> int {
      if (next_len + n > arena_cap) return set_last_error(TESSA_ERR_PARTITION, "subtree arena exceeded");
      HNode h = proto;
      h.off = (uint32_t)next_len;
      h.n = n;
      *dest = next_len;
      next_len += n;
      next_nodes.push_back(h);
      return TESSA_OK;
    };
    for (size_t q = 0; q < nodes.size(); ++q) {
      const HNode& nd = nodes[q];
      if (kind[q] == kLeafNode) {
        uint64_t at;
        if (!leaf_alloc(nd.n, &at)) return set_last_error(TESSA_ERR_PARTITION, "subtree leaf_rows capacity exceeded");
        leaves.push_back(LeafEnt{at, nd.n, nd.task});
        sc.push_back(NodeDesc{nd.off, nd.n, nd.task, 0, 0, 0, nd.depth, kCopyLeaf, nd.seed, dests.size()});
        dests.push_back(at | kLeafBit);
        continue;
      }
      if (kind[q] == kSmall) {
        uint64_t at;
        const uint32_t lf = fs;  // reservation: every row in at most fanout_second children
        if (!leaf_alloc((uint64_t)nd.n * lf, &at))
          return set_last_error(TESSA_ERR_PARTITION, "subtree leaf_rows capacity exceeded");
        sm.push_back(NodeDesc{nd.off, nd.n, nd.task, 0, 0, 0, nd.depth, 0, nd.seed, at});
        sm_leaf_pos.push_back(leaves.size());
        stats->small_nodes++;
        continue;
      }
      // large
      const uint32_t* c = counts.data() + li * kSlots;
      li++;
      uint32_t nonempty = 0, max_child = 0;
      for (uint32_t s = 0; s < nd.num; ++s)
        if (c[s]) {
          nonempty++;
          max_child = std::max(max_child, c[s]);
        }
      const bool split = nonempty > 1u && meaningful_split(nd.n, max_child, a.leaf_max);
      uint32_t retry_max = nd.n < 2u ? 2u : nd.n;
      if (retry_max > kSlots) retry_max = kSlots;
      NodeDesc plan{nd.off, nd.n, nd.task, nd.num, nd.attempt, nd.lf, nd.depth, kSplit, nd.seed, dests.size()};
      uint64_t dst[kSlots];
      memset(dst, 0, sizeof dst);
      if (!split && (nd.attempt == 0 || nd.num < retry_max)) {
        uint32_t next_num = nd.num;
        if (nd.attempt > 0) {
          const uint32_t dbl = nd.num << 1;
          next_num = (dbl > nd.num && dbl < retry_max) ? dbl : retry_max;
        }
        if (next_num > retry_max) next_num = retry_max;
        HNode again = nd;
        again.attempt = nd.attempt + 1;
        again.num = next_num;
        int rc = push_next(again, nd.n, &dst[0]);
        if (rc) return rc;
        plan.mode = kCopyNext;
        stats->retries++;
      } else {
        uint32_t nchild = nd.num;
        uint32_t len2[2] = {(nd.n + 1u) >> 1, nd.n >> 1};
        if (!split) {
          plan.mode = kBalanced;
          nchild = 2;
          stats->balanced++;
        }
        for (uint32_t ci = 0; ci < nchild; ++ci) {
          const uint32_t len = split ? c[ci] : len2[ci];
          if (len == 0) continue;
          if (len <= a.leaf_max) {
            uint64_t at;
            if (!leaf_alloc(len, &at)) return set_last_error(TESSA_ERR_PARTITION, "subtree leaf_rows capacity exceeded");
            leaves.push_back(LeafEnt{at, len, nd.task});
            dst[ci] = at | kLeafBit;
          } else if (nd.depth + 1u >= a.max_depth) {
            return set_last_error(TESSA_ERR_PARTITION, "subtree child above leaf_max at max_depth (oversized terminal)");
          } else {
            HNode ch{nd.task, 0, len, nd.depth + 1u, 0u, 0u, 0u, child_seed(nd.seed, ci, len)};
            int rc = push_next(ch, len, &dst[ci]);
            if (rc) return rc;
          }
        }
      }
      sc.push_back(plan);
      // destinations the scatter reads: one (copy), two (balanced) or one per leader slot
      const uint32_t ndst = plan.mode == kCopyNext ? 1u : (plan.mode == kBalanced ? 2u : nd.num);
      dests.insert(dests.end(), dst, dst + ndst);
    }

    stats->host_decide_ms += ms_since(t_decide);
    // ---- scatter (leaf-all and large nodes) and the small path
    if (!sc.empty()) {
      ST_ALLOC(S->nodes, sc.size() * sizeof(NodeDesc));
      ST_ALLOC(S->dests, dests.size() * 8);
      S->stage_scatter.add(S->nodes.ptr, sc.data(), sc.size() * sizeof(NodeDesc));
      S->stage_scatter.add(S->dests.ptr, dests.data(), dests.size() * 8);
      ST_CUDA(S->stage_scatter.flush(st));
      ST_CUDA(cudaEventRecord(S->ev[2], st));
      scatter_kernel<<<(unsigned)sc.size(), 256, 0, st>>>(S->nodes.as<NodeDesc>(), S->dests.as<uint64_t>(),
                                                         S->cur.as<uint32_t>(), S->slots.as<uint32_t>(),
                                                         a.task_members, S->task_off.as<uint64_t>(),
                                                         S->next.as<uint32_t>(), a.leaf_rows);
      ST_CUDA(cudaGetLastError());
      ST_CUDA(cudaEventRecord(S->ev[3], st));
      stats->launches++;
    }
    if (!sm.empty()) {
      ST_ALLOC(S->small_nodes, sm.size() * sizeof(NodeDesc));
      ST_ALLOC(S->tables, sm.size() * kTab * 4);
      S->stage_small.add(S->small_nodes.ptr, sm.data(), sm.size() * sizeof(NodeDesc));
      ST_CUDA(S->stage_small.flush(st));
      SmallParams sp{};
      sp.nodes = S->small_nodes.as<NodeDesc>();
      sp.cur = S->cur.as<uint32_t>();
      sp.task_members = a.task_members;
      sp.task_off = S->task_off.as<uint64_t>();
      sp.codes = a.codes;
      sp.scales = a.scales;
      sp.norms = a.sq8_norms;
      sp.padded_dim = a.padded_dim;
      sp.leaf_max = a.leaf_max;
      sp.leaf_min = a.leaf_min;
      sp.max_leaders = max_leaders;
      sp.fanout_second = fs;
      sp.root_depth = a.root_depth;
      sp.psamp = a.psamp_fraction;
      sp.leaf_rows = a.leaf_rows;
      sp.tables = S->tables.as<uint32_t>();
      sp.err = d_err;
      ST_CUDA(cudaEventRecord(S->ev[4], st));
      small_kernel<<<(unsigned)sm.size(), 256, small_smem, st>>>(sp);
      ST_CUDA(cudaGetLastError());
      ST_CUDA(cudaEventRecord(S->ev[5], st));
      stats->launches++;
      std::vector<uint32_t> tab(sm.size() * kTab);
      if (!S->h_tables.ensure(tab.size() * 4) || !S->h_bits.ensure(8))
        return set_last_error(TESSA_ERR_OOM, "subtree pinned staging allocation failed");
      ST_CUDA(cudaMemcpyAsync(S->h_tables.p, S->tables.ptr, tab.size() * 4, cudaMemcpyDeviceToHost, st));
      ST_CUDA(cudaMemcpyAsync(S->h_bits.p, d_err, 4, cudaMemcpyDeviceToHost, st));
      ST_CUDA(cudaStreamSynchronize(st));
      const uint32_t bits = *S->h_bits.as<uint32_t>();
      memcpy(tab.data(), S->h_tables.p, tab.size() * 4);
      if (bits) return set_last_error(TESSA_ERR_BAD_TASK, "subtree small-node partition failed");
      // insert each small node's leaves at its place in the list (back to front
      // so earlier insertion points stay valid)
      for (size_t j = sm.size(); j-- > 0;) {
        const uint32_t* tb = tab.data() + j * kTab;
        std::vector<LeafEnt> ins;
        for (uint32_t cidx = 0; cidx < tb[0]; ++cidx)
          ins.push_back(LeafEnt{sm[j].out + tb[1 + 2 * cidx], tb[2 + 2 * cidx], sm[j].task});
        leaves.insert(leaves.begin() + (ptrdiff_t)sm_leaf_pos[j], ins.begin(), ins.end());
      }
    }
    if (a.leaf_codes && leaf_used > leaf_round0) {
      // this round's leaves are final: copy their codes while the host decides
      ST_CUDA(cudaEventRecord(S->round_done, st));
      ST_CUDA(cudaStreamWaitEvent(S->side, S->round_done, 0));
      const int grc = launch_gather_rows(a.codes, a.leaf_rows + leaf_round0, leaf_used - leaf_round0, a.padded_dim,
                                         a.resident_rows, a.leaf_codes + leaf_round0 * a.padded_dim, sm_count,
                                         S->side);
      if (grc != TESSA_OK) return set_last_error(grc, "subtree leaf-code copy launch failed");
      stats->launches++;
    }
    const auto t_end = clk::now();
    ST_CUDA(cudaStreamSynchronize(st));
    stats->sync_wait_ms += ms_since(t_end);
    if (!sc.empty()) stats->scatter_ms += elapsed(2, 3);
    if (!sm.empty()) stats->small_ms += elapsed(4, 5);
    std::swap(S->cur, S->next);
    nodes.swap(next_nodes);
  }

  if (leaves.size() > a.leaf_capacity)
    return set_last_error(TESSA_ERR_PARTITION, "subtree leaf table capacity exceeded");
  for (size_t l = 0; l < leaves.size(); ++l) {
    a.leaf_starts[l] = leaves[l].start;
    a.leaf_sizes[l] = leaves[l].size;
    if (a.leaf_tasks) a.leaf_tasks[l] = leaves[l].task;
  }
  stats->leaf_count = leaves.size();
  stats->leaf_rows_used = leaf_used;
  stats->wall_ms = std::chrono::duration<float, std::milli>(std::chrono::steady_clock::now() - wall0).count();
  return TESSA_OK;
}

}  // namespace tessa
