// SQ8 leaf all-pairs evaluation with fused per-row bounded top-k, sm_100a.
//
// Reference semantics (wbh1765091327/SHEAR, CB = shear-core/src/algorithm/
// pipnn/compute_backend.rs):
//   * candidates of row r are the other members of its leaf, taken in
//     ascending member position, skipping columns whose local id equals the
//     row's (CB:9569-9650, CB:10046-10096);
//   * distance = gpu_persistent_sq_int8_l2_from_dot (CB:8987-9002);
//   * each candidate goes through gpu_persistent_insert_topk_candidate_fp32
//     (CB:7229-7259) into a k-slot list initialised to (FLT_MAX, 0xffffffff);
//   * output ids are the candidates' global ids, written at (start + r) * k.
//
// B200 design (one persistent CTA per SM, 192 threads):
//   warp 0      TMA producer: A = 128 leaf rows x padded_dim (resident for the
//               tile), B = 256-column chunks streamed in 128-byte K slabs
//               through a ring of shared-memory stages (SWIZZLE_128B).
//   warp 1      TMEM owner + single-thread tcgen05.mma issuer (kind::i8,
//               M=128, N=256, K=32, int32 accumulators), double-buffered in
//               TMEM (2 x 256 columns) so the epilogue of chunk c overlaps the
//               MMAs of chunk c+1.
//   warps 2..5  epilogue: thread t owns TMEM lane (= leaf row) t; it reads 32
//               accumulator columns per tcgen05.ld, turns them into the exact
//               reference distances, filters them against its list's worst
//               entry (with a margin that covers the list's possible upward
//               creep under the eps rule), stashes survivors in shared memory
//               in column order and then inserts them with the reference's
//               exact insertion rule held in registers.
// The distance matrix never leaves the SM.
#include "common.cuh"
#include "kernels.h"

namespace tessa {
namespace leaf {

constexpr uint32_t kBM = 128;          // rows per tile (TMEM lanes)
constexpr uint32_t kBN = 256;          // columns per chunk (MMA N)
constexpr uint32_t kSlab = 128;        // K bytes per TMA box (one 128B swizzle atom)
constexpr uint32_t kMmaK = 32;         // K per tcgen05.mma kind::i8
constexpr uint32_t kThreads = 192;
constexpr uint32_t kEpiThreads = 128;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kASlabBytes = kBM * kSlab;   // 16 KiB
constexpr uint32_t kBStageBytes = kBN * kSlab;  // 32 KiB
constexpr uint32_t kGroup = 32;                 // columns per tcgen05.ld
constexpr uint32_t kMaxBStages = 6;
constexpr uint32_t kMetaBytes = 2u * kBN * 16u;              // 2 chunk buffers of (s, n, lid, gid)
constexpr uint32_t kStashDBytes = 4u * kGroup * 32u * 4u;    // per epilogue warp: 32 entries x 32 lanes
constexpr uint32_t kStashCBytes = 4u * kGroup * 32u;
constexpr uint32_t kBarBytes = 256u;
constexpr uint32_t kSmemLimit = 232448u;  // 227 KiB opt-in per block

// Upward creep bound of the list's last distance while one group of at most
// 32 candidates is inserted: each insertion can raise it by at most the tie
// eps, so survivors are filtered against worst + 33 * eps.
constexpr float kFilterMargin = 33.0f * 2.0e-5f;

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
  uint32_t* out_ids;
  float* out_dists;
  uint32_t* err_word;
  uint64_t timeout_ns;
};

struct Smem {
  uint8_t* a;
  uint8_t* b;
  uint4* meta;
  float* stash_d;
  uint8_t* stash_c;
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
  return 1024u + num_slabs * kASlabBytes + num_bstages * kBStageBytes + kMetaBytes + kStashDBytes +
         kStashCBytes + kBarBytes;
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
  s.stash_d = reinterpret_cast<float*>(p);
  p += kStashDBytes;
  s.stash_c = p;
  p += kStashCBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(p);
  s.a_full = bars + 0;
  s.a_empty = bars + 1;
  s.b_full = bars + 2;
  s.b_empty = bars + 2 + kMaxBStages;
  s.t_full = bars + 2 + 2 * kMaxBStages;
  s.t_empty = bars + 4 + 2 * kMaxBStages;
  s.mma_done = bars + 6 + 2 * kMaxBStages;
  s.tmem_slot = reinterpret_cast<uint32_t*>(bars + 7 + 2 * kMaxBStages);
  s.abort_flag = s.tmem_slot + 1;
  s.epi_stop = s.tmem_slot + 2;
  return s;
}

// Exact reference insertion (CB:7229-7259) into a register list of KMAX slots.
// The live list occupies slots [KMAX-k, KMAX); slots below hold sentinels that
// nothing is "better" than, so the shift stops there exactly as the
// reference's loop stops at position 0 of a k-slot list.
template <int KMAX>
__device__ __forceinline__ void insert_exact(float d, uint32_t id, float (&bd)[KMAX], uint32_t (&bi)[KMAX]) {
  if (!stable_better(d, id, bd[KMAX - 1], bi[KMAX - 1])) return;
  // Branch-free shift: `run` stays true while the candidate is still moving up.
  bool run = true;
#pragma unroll
  for (int j = KMAX - 1; j >= 1; --j) {
    float delta = __fsub_rn(d, bd[j - 1]);
    bool tie = fabsf(delta) <= 2.0e-5f;
    bool better = (tie & (id < bi[j - 1])) | ((!tie) & (d < bd[j - 1]));
    bool b = run & better;
    float nd = b ? bd[j - 1] : (run ? d : bd[j]);
    uint32_t ni = b ? bi[j - 1] : (run ? id : bi[j]);
    bd[j] = nd;
    bi[j] = ni;
    run = b;
  }
  if (run) {
    bd[0] = d;
    bi[0] = id;
  }
}

__device__ __forceinline__ uint4 load_meta(const Params& p, uint64_t start, uint32_t cnt, uint32_t col) {
  if (col >= cnt) return make_uint4(0u, 0u, 0xffffffffu, 0xffffffffu);
  uint32_t lid = __ldg(p.members + start + col);
  float s = __ldg(p.scales + lid);
  float n = __ldg(p.norms + lid);
  uint32_t gid = __ldg(p.global_ids + lid);
  return make_uint4(__float_as_uint(s), __float_as_uint(n), lid, gid);
}

template <int KMAX>
__global__ void __launch_bounds__(kThreads, 1)
    leaf_topk_sq8_kernel(const __grid_constant__ CUtensorMap tmap_a,
                         const __grid_constant__ CUtensorMap tmap_b, const Params p) {
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
    for (uint32_t i = 0; i < 2; ++i) {
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
          tma_load_2d(&tmap_a, s.a + sl * kASlabBytes, s.a_full, (int32_t)(sl * kSlab),
                      (int32_t)(start + t.y));
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
          uint32_t buf = acc & 1u, use = acc >> 1;
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
    const uint32_t ew = warp - 2;             // epilogue warp 0..3
    const uint32_t quad = warp & 3u;          // TMEM lane quadrant this warp may access
    const uint32_t et = threadIdx.x - 64;     // 0..127
    const uint32_t row_in_tile = quad * 32 + lane;
    float* stash_d = s.stash_d + ew * (kGroup * 32);
    uint8_t* stash_c = s.stash_c + ew * (kGroup * 32);
    uint32_t acc = 0;
    bool stop = false;
    for (uint32_t tile = blockIdx.x; tile < p.num_tiles && !stop; tile += gridDim.x) {
      uint2 t = p.tiles[tile];
      uint64_t start = p.leaf_starts[t.x];
      uint32_t cnt = p.leaf_sizes[t.x];
      uint32_t row = t.y + row_in_tile;
      bool valid = row < cnt;
      uint32_t lid_i = 0xffffffffu;
      float s_i = 0.f, n_i = 0.f;
      if (valid) {
        lid_i = __ldg(p.members + start + row);
        s_i = __ldg(p.scales + lid_i);
        n_i = __ldg(p.norms + lid_i);
      }
      float bd[KMAX];
      uint32_t bi[KMAX];
#pragma unroll
      for (int j = 0; j < KMAX; ++j) {
        bool live = j >= KMAX - (int)p.k;
        bd[j] = live ? 3.402823466e+38F : -INFINITY;
        bi[j] = live ? 0xffffffffu : 0u;
      }
      uint32_t nchunks = (cnt + kBN - 1) / kBN;
      // chunk 0 metadata
      s.meta[et] = load_meta(p, start, cnt, et);
      s.meta[et + 128] = load_meta(p, start, cnt, et + 128);
      __syncwarp();
      named_bar_sync(1, kEpiThreads);
      for (uint32_t c = 0; c < nchunks; ++c, ++acc) {
        uint4* meta = s.meta + (c & 1u) * kBN;
        uint4 nm0 = make_uint4(0, 0, 0, 0), nm1 = nm0;
        if (c + 1 < nchunks) {
          nm0 = load_meta(p, start, cnt, (c + 1) * kBN + et);
          nm1 = load_meta(p, start, cnt, (c + 1) * kBN + et + 128);
        }
        uint32_t buf = acc & 1u, use = acc >> 1;
        // Warp-uniform bounded wait: tcgen05.ld below is warp-collective.
        bool ok = true;
        if (lane == 0) ok = mbar_wait(&s.t_full[buf], use & 1u, abort_flag, p.err_word, p.timeout_ns);
        ok = __shfl_sync(0xffffffffu, ok ? 1u : 0u, 0) != 0u;
        if (ok) {
          tc_fence_after();
#pragma unroll 1
          for (uint32_t g = 0; g < kBN / kGroup; ++g) {
            uint32_t v[32];
            tmem_ld_32x32b_x32(tmem_base + ((quad * 32u) << 16) + buf * kBN + g * kGroup, v);
            tmem_ld_wait();
            float thr = __fadd_rn(bd[KMAX - 1], kFilterMargin);
            uint32_t n_st = 0;
#pragma unroll
            for (uint32_t cc = 0; cc < kGroup; ++cc) {
              uint4 m = meta[g * kGroup + cc];
              float d = sq8_l2_from_dot((int)v[cc], s_i, n_i, __uint_as_float(m.x), __uint_as_float(m.y));
              bool pass = valid && (d <= thr) && (m.z != lid_i) && (m.z != 0xffffffffu);
              if (pass) {
                stash_d[n_st * 32 + lane] = d;
                stash_c[n_st * 32 + lane] = (uint8_t)(g * kGroup + cc);
                ++n_st;
              }
            }
#pragma unroll 1
            for (uint32_t e = 0; e < n_st; ++e) {
              float d = stash_d[e * 32 + lane];
              uint32_t col = stash_c[e * 32 + lane];
              insert_exact<KMAX>(d, meta[col].w, bd, bi);
            }
            __syncwarp();
          }
          tc_fence_before();
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.t_empty[buf]);
        if (c + 1 < nchunks) {
          uint4* nxt = s.meta + ((c + 1) & 1u) * kBN;
          nxt[et] = nm0;
          nxt[et + 128] = nm1;
        }
        // Uniform stop decision for the four epilogue warps (named barrier
        // below must see all of them every chunk).
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
#pragma unroll
        for (int j = 0; j < KMAX; ++j) {
          int slot = j - (KMAX - (int)p.k);
          if (slot >= 0) {
            p.out_ids[out + slot] = bi[j];
            p.out_dists[out + slot] = bd[j];
          }
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

template <int KMAX>
static cudaError_t launch_leaf_k(const LeafLaunch& L, const CUtensorMap& ta, const CUtensorMap& tb,
                                 const leaf::Params& prm, uint32_t smem, cudaStream_t stream) {
  auto kern = leaf::leaf_topk_sq8_kernel<KMAX>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  uint32_t grid = L.num_tiles < (uint32_t)L.sm_count ? L.num_tiles : (uint32_t)L.sm_count;
  if (grid == 0) return cudaSuccess;
  kern<<<grid, leaf::kThreads, smem, stream>>>(ta, tb, prm);
  return cudaGetLastError();
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
  prm.out_ids = L.out_ids;
  prm.out_dists = L.out_dists;
  prm.err_word = L.d_err;
  prm.timeout_ns = L.timeout_ns;
  uint32_t smem = leaf::smem_bytes(slabs, (uint32_t)nst);
  cudaError_t e;
  if (L.k <= 4)
    e = launch_leaf_k<4>(L, ta, tb, prm, smem, stream);
  else if (L.k <= 8)
    e = launch_leaf_k<8>(L, ta, tb, prm, smem, stream);
  else if (L.k <= 16)
    e = launch_leaf_k<16>(L, ta, tb, prm, smem, stream);
  else
    e = launch_leaf_k<32>(L, ta, tb, prm, smem, stream);
  return e == cudaSuccess ? TESSA_OK : TESSA_ERR_CUDA;
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
