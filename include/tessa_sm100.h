/*
 * tessa_sm100.h -- C ABI of the B200 (sm_100a) TESSA hot-path library
 * (libtessa_sm100.so).
 *
 * The library replaces the NVRTC/cudarc leaf and assignment kernel bindings of
 * SHEAR (wbh1765091327/SHEAR).  Reference paths below are relative to that
 * project's root; CB = shear-core/src/algorithm/pipnn/compute_backend.rs,
 * P = shear-core/src/algorithm/pipnn/.
 *
 * Conventions
 *  - Every function returns TESSA_OK (0) or a negative TESSA_ERR_* code; nothing
 *    aborts or unwinds across the ABI.  tessa_strerror() names a code and
 *    tessa_last_error_message() gives the detail of the calling thread's last
 *    failure.
 *  - "device pointer" arguments point to CUDA device memory on the context's
 *    device; "host pointer" arguments point to ordinary (pageable or pinned)
 *    host memory owned by the caller.  The library owns every buffer it
 *    allocates (device scratch, pinned staging) and frees it in the matching
 *    destroy call.
 *  - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *  - A context is bound to one device and is not thread-safe: use one context
 *    per GPU per host thread (the reference serialises its CUDA engine behind a
 *    mutex, CB:34666).
 *  - Distances follow the reference bit for bit: SQ8 leaf distances are
 *    rn(rn(n_i+n_j) + rn(-2*rn(rn(s_i*s_j)*dot))) clamped at 0 (CB:8987-9002);
 *    leaf lists use the stable eps/id order of CB:7229-7259.
 */
#ifndef TESSA_SM100_H
#define TESSA_SM100_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define TESSA_API __attribute__((visibility("default")))
#else
#define TESSA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* 1: leaf, quantize, assignment, replay; 2: + host pipeline knob, global D0, candidate
 * edges, capture digests, graph search (additive); 3: + subtree partition (additive). */
#define TESSA_ABI_VERSION 5

#define TESSA_OK 0
#define TESSA_ERR_INVALID_ARG (-1)  /* malformed sizes, null pointers, k out of range */
#define TESSA_ERR_CUDA (-2)         /* a CUDA runtime/driver call failed */
#define TESSA_ERR_OOM (-3)          /* device or pinned allocation failed */
#define TESSA_ERR_TIMEOUT (-4)      /* a bounded device wait expired (kernel gave up) */
#define TESSA_ERR_BAD_ROW (-5)      /* a member/leader id is outside the resident rows */
#define TESSA_ERR_UNSUPPORTED (-6)  /* shape or mode this build does not implement */
#define TESSA_ERR_NONFINITE (-7)    /* non-finite input to the SQ8 quantizer */
#define TESSA_ERR_NO_DEVICE (-8)    /* no sm_100 device / extension not usable */
#define TESSA_ERR_BAD_TASK (-9)     /* malformed task descriptor seen on the device */
#define TESSA_ERR_AGAIN (-11)       /* not now: no free submission slot, or the submission is still running */
#define TESSA_ERR_PARTITION (-10)   /* the subtree partition cannot finish: a node above leaf_max at max_depth
                                       (GPU_PERSISTENT_OVERSIZED_TERMINAL_NODE, CB:4849) or output capacity */

/* Largest leaf k (CB:4890 GPU_PERSISTENT_LEAF_DCO_MAX_SURVIVORS). */
#define TESSA_MAX_LEAF_K 32
/* Largest assignment fan-out r_h (CB:15784-15786). */
#define TESSA_MAX_RH 4
/* Largest padded SQ8 dimension the leaf kernel accepts (shared-memory bound). */
#define TESSA_MAX_PADDED_DIM 1024
/* Largest leaf (member rows) the leaf kernel accepts. */
#define TESSA_MAX_LEAF_ROWS 65535

typedef struct tessa_ctx tessa_ctx;
typedef struct tessa_replay_session tessa_replay_session;

/* ---------------------------------------------------------------- misc --- */

TESSA_API int tessa_abi_version(void);
TESSA_API const char* tessa_strerror(int code);
/* Detail of the last failure on the calling thread ("" if none). */
TESSA_API const char* tessa_last_error_message(void);

/* Replaces CudaComputeBackend::new / validate_gpu_subtree_hardware
 * (CB:3693-3884 trait, CB:34654-34662 SM check): binds device `device`,
 * verifies it is sm_100 and prepares library state. */
TESSA_API int tessa_create(int device, tessa_ctx** out);
TESSA_API void tessa_destroy(tessa_ctx* ctx);
TESSA_API int tessa_ctx_device(const tessa_ctx* ctx);
/* Device bytes the context currently holds in scratch and staging buffers
 * (grow-only; freed by tessa_destroy) -- the quantity the task former's
 * admission model bounds. */
TESSA_API int tessa_ctx_device_bytes(const tessa_ctx* ctx, uint64_t* bytes);

/* ------------------------------------------------------- SQ8 quantizer --- */

/* Per-row symmetric int8 quantization, bit-exact with the reference CPU
 * quantizer quantize_sq_int8_matrix_with_bits (P/dco_sq_int8.rs:1331-1375,
 * 1431-1466), which the reference replay uses (P/tessa_replay.rs:1291-1296):
 *   norm  = sequential f32 sum of x*x; scale = max|x| / (2^(bits-1)-1) (1 if 0);
 *   code  = clamp(round_half_away(x/scale)), zero-padded to padded_dim =
 *           ceil(dim/k_align)*k_align.
 * Replaces sq8_quantize_rows_kernel (CB:17955-18014), whose tree-reduced norm
 * does not match the CPU bits.  Device pointers; codes is rows x padded_dim. */
TESSA_API int tessa_quantize_sq8(tessa_ctx* ctx, const float* x, uint64_t rows, uint32_t dim,
                       uint32_t k_align, uint32_t bits, int8_t* codes, float* scales, float* norms,
                       void* stream);

/* Host-buffer variant (copies in and out inside the call). */
TESSA_API int tessa_quantize_sq8_host(tessa_ctx* ctx, const float* x, uint64_t rows, uint32_t dim,
                            uint32_t k_align, uint32_t bits, int8_t* codes, float* scales,
                            float* norms);

/* ------------------------------------------------------- SQ8 leaf top-k --- */

/* A batch of leaves, laid out as the reference replay lays them out
 * (TessaLeafLayout, P/tessa_replay.rs:1045-1050; leaf descriptors CB:35189-35230):
 * leaf l owns leaf_members[leaf_starts[l] .. leaf_starts[l] + leaf_sizes[l]),
 * each entry a local resident row id; output row r of leaf l is written at
 * (leaf_starts[l] + r) * k in topk_ids / topk_dists. */
typedef struct tessa_leaf_args {
  /* resident rows, indexed by local id (device pointers) */
  const int8_t* codes;          /* resident_rows x padded_dim, zero padded */
  const float* scales;          /* SQ8 scales */
  const float* norms;           /* SQ8 norms (CB:35094-35098 passes sq8_norms) */
  const uint32_t* global_ids;   /* output id of each resident row */
  uint64_t resident_rows;
  uint32_t padded_dim;          /* multiple of 16, <= TESSA_MAX_PADDED_DIM */
  uint32_t k;                   /* 1 .. TESSA_MAX_LEAF_K */
  /* leaf layout */
  const uint32_t* leaf_members; /* device pointer, leaf_rows entries (entries in no leaf are never
                                   used; those at or above resident_rows are not read) */
  const uint64_t* leaf_starts;  /* HOST pointer, leaf_count entries */
  const uint64_t* leaf_sizes;   /* HOST pointer, leaf_count entries */
  uint64_t leaf_count;
  uint64_t leaf_rows;           /* total member entries */
  /* outputs (device pointers, leaf_rows * k entries each) */
  uint32_t* topk_ids;
  float* topk_dists;
  /* Optional (may be NULL): codes already in leaf order, row p = codes row
   * leaf_members[p], leaf_rows x padded_dim.  When NULL the library gathers
   * them into its own device scratch (leaf_rows * padded_dim bytes). */
  const int8_t* leaf_ordered_codes;
} tessa_leaf_args;

/* All-pairs SQ8 leaf evaluation with per-row bounded top-k: int8 tcgen05 GEMM
 * with int32 accumulation in TMEM fed by TMA, fused with the reference's
 * per-row sorted insertion (ascending member order, self skipped by local id,
 * CB:9569-9650), so no distance matrix reaches HBM.  Replaces
 * gpu_persistent_subtree_topk_only's SQ8 executors (CB:16146, CB:9364,
 * CB:10389) as launched by TessaCudaReplaySession::launch_leaf
 * (CB:35026-35152).  Rows without k candidates keep (FLT_MAX, 0xffffffff)
 * in their tail slots.  Device scratch held by the context, grown on demand:
 * the optional leaf-ordered codes (above), the tile table, the exact-fallback
 * row list (8 bytes per row) and, for padded_dim <= 1024, a per-row zone dump
 * of 8 * min(k + 7, 48) rounded down to even, plus 130, bytes per leaf row (434
 * at k = 32: the leaf kernel's candidates near each row's k-th distance, read
 * back by its finishing kernel). */
TESSA_API int tessa_leaf_topk_sq8(tessa_ctx* ctx, const tessa_leaf_args* args, void* stream);

/* Host-buffer variant: every pointer of `args` (including leaf_members and the
 * outputs) is a HOST pointer; the call uploads, runs and downloads.  This is
 * the form the compute-backend trait method
 * process_quantized_subtree_l2_compact_topk (CB:3693-3884) binds. */
TESSA_API int tessa_leaf_topk_sq8_host(tessa_ctx* ctx, const tessa_leaf_args* args);

/* Batch size (bytes of codes) of the host-buffer call's copy/compute pipeline,
 * used when leaf_members is the identity and the leaves are in ascending,
 * disjoint row order: batch b's upload, leaf kernel and download overlap
 * those of its neighbours.  0 restores the default (128 MiB).  A library
 * tuning knob with no reference counterpart; results do not depend on it. */
TESSA_API int tessa_set_host_batch_bytes(tessa_ctx* ctx, uint64_t bytes);

/* Rows of the context's last leaf call whose lists depended on insertion order
 * (eps-tie chains) and were recomputed with the exact sequential rule -- the
 * counterpart of the reference's leaf_exact_fallback_rows counter
 * (P/tessa_replay.rs:155-188; here it is a diagnostic, not an error). */
TESSA_API int tessa_leaf_last_fallback_rows(const tessa_ctx* ctx, uint64_t* rows);
/* Which form of the column-split leaf kernel a context uses: 1 (default) --
 * one CTA per 128-row tile loading every chunk of B columns; 0 -- pairs of
 * CTAs on neighbouring SMs (a cluster of two) share each chunk, one 256-row
 * MMA (tcgen05 cta_group::2) over two 128-row tiles of the same leaf, each
 * CTA loading half of the chunk.  Both give the same lists bit for bit; the
 * pair form halves the B traffic but runs its two CTAs in lock step, which
 * measured slower on epilogue-bound leaves.  It needs whole-batch calls and
 * falls back to the single form when no cluster can be placed.  Returns
 * TESSA_ERR_INVALID_ARG for other modes. */
TESSA_API int tessa_set_leaf_kernel(tessa_ctx* ctx, uint32_t mode);

/* Size of the static device scratch of tessa_leaf_topk_sq8_noalloc (64 MiB). */
#define TESSA_NOALLOC_SCRATCH_BYTES (64u << 20)

/* Allocation-free form of tessa_leaf_topk_sq8 (this entry point has no
 * counterpart in the reference).  For callers that must not allocate device
 * memory: hosts whose allocator owns the whole device, latency-critical
 * threads where cudaMalloc/cudaFree (which can synchronise the device) are not
 * allowed, embedders that fix their footprint at load time.  Same arguments
 * and results as tessa_leaf_topk_sq8 (device pointers, HOST leaf layout), on
 * the current device, but no context: its scratch (tile table, error word,
 * exact-fallback row list and, when leaf_ordered_codes is NULL, the
 * leaf-ordered copy of the codes) lives in
 * one static device array of TESSA_NOALLOC_SCRATCH_BYTES that every GPU loading
 * the library holds until exit.  Batches needing more scratch are rejected
 * with TESSA_ERR_UNSUPPORTED.  The first call on a device resolves the array's
 * address (make it before any stream capture) and keeps it for the process; a
 * device reset makes it stale, so do not call this again after one.  All calls
 * share the array and
 * leave their contents in it; calls whose GPU work overlaps race and must be
 * serialised by the caller.  Returns after the work has completed. */
TESSA_API int tessa_leaf_topk_sq8_noalloc(const tessa_leaf_args* args, void* stream);

/* ------------------------------------------------------------ assignment --- */

/* Frozen assignment tasks in the replay layout (TessaAssignmentLayout,
 * P/tessa_replay.rs:1036-1043; kernel arguments CB:15729-15758). */
typedef struct tessa_assign_args {
  const float* x;              /* resident_rows x dim raw vectors (FP32 modes) */
  const float* raw_norms;      /* FP32-mode norms */
  const int8_t* codes;         /* resident_rows x padded_dim (SQ8 modes) */
  const float* scales;
  const float* sq8_norms;
  const uint32_t* global_ids;
  uint64_t resident_rows;
  uint32_t dim;
  uint32_t padded_dim;
  const uint32_t* members;
  const uint32_t* leaders;
  const uint32_t* task_member_offsets;
  const uint32_t* task_member_counts;
  const uint32_t* task_leader_offsets;
  const uint32_t* task_leader_counts;
  const uint32_t* task_rh;
  const uint64_t* task_output_offsets;
  uint32_t task_count;
  uint64_t member_rows;        /* total member entries over all tasks */
  uint32_t* out_ids;           /* output_len entries */
  float* out_dists;
} tessa_assign_args;

/* Distance source of an assignment call. */
#define TESSA_ASSIGN_FP32 0u  /* A0: sequential FP32 dot, CB:13646-13896 / CB:6436-6444 */
#define TESSA_ASSIGN_SQ8 2u   /* SQ8 int8 dot, n_p+n_l-2*s_p*s_l*dot, CB:14676-14678 */

/* Per-row best r_h <= 4 leaders (local fan-out 4, CB:15808) with the
 * reference's splitmix64 tie keys (CB:6510-6578); output id =
 * global_ids[leader].  All pointers are device pointers except the task
 * arrays, which are HOST pointers (the library uploads them). */
TESSA_API int tessa_assign(tessa_ctx* ctx, uint32_t source, const tessa_assign_args* args, void* stream);

/* ------------------------------------------------------------ global D0 --- */

/* Global-D0 SQ8 staging, the compute-backend trait method
 * quantize_sq8_and_assign_global_d0 (trait CB:3828-3837; CUDA implementation
 * CB:24281-24760 with kernels CB:17955-18112, 18114, 18446; CPU reference
 * quantize_sq8_and_assign_global_d0_reference, P/dco_sq_int8.rs:1929-2070,
 * called from P/rbc_partition.rs:8429).  Quantizes a batch of raw rows to SQ8
 * (CPU quantizer bits, P/dco_sq_int8.rs:1331-1466) and assigns every row to
 * its fanout_top nearest global D0 leaders by SQ8 distance (CB:8987-9002
 * rounding), ordered by the stable eps/id rule on (distance, leader id)
 * (P/mod.rs:417-428).  Output fragment (row, slot) = (child_ids, point_ids)
 * at row * fanout_top + slot: the leader INDEX (0..leader_count) and the
 * row's global id, best leader first -- the reference's D0AssignmentFragment
 * list (P/dco_sq_int8.rs:2055-2060) as two arrays. */
typedef struct tessa_d0_args {
  const float* raw_vectors;     /* rows x dim f32, row-major */
  const uint32_t* global_ids;   /* rows */
  uint64_t rows;
  uint32_t dim;                 /* padded_dim = ceil(dim / 16) * 16 */
  uint32_t fanout_top;          /* 1 .. min(32, leader_count) */
  const uint32_t* leader_ids;   /* leader_count global D0 leader ids (tie order) */
  const float* leader_vectors;  /* leader_count x dim f32; used when leader_codes is NULL */
  const int8_t* leader_codes;   /* optional SQ8 leader payload, leader_count x padded_dim */
  const float* leader_scales;   /* with leader_codes: leader_count */
  const float* leader_norms;    /* with leader_codes: leader_count */
  uint32_t leader_count;
  int8_t* codes;                /* out: rows x padded_dim */
  float* scales;                /* out: rows */
  float* norms;                 /* out: rows */
  uint32_t* child_ids;          /* out: rows x fanout_top leader indices */
  uint32_t* point_ids;          /* out: rows x fanout_top (= global_ids[row]) */
  float* dists;                 /* optional out: rows x fanout_top SQ8 distances (NULL = not written) */
} tessa_d0_args;

/* Phase times of the context's last D0 call, from CUDA events on its stream --
 * the device-side fields of the reference's SqGpuD0StagingProfile
 * (P/dco_sq_int8.rs:411-436: gpu_quantize_wall, leader_quantize_wall,
 * d0_assign_distance_kernel_wall, d0_assign_merge_kernel_wall). */
typedef struct tessa_d0_profile {
  double leader_quantize_ms;    /* 0 when a leader payload was given */
  double quantize_ms;           /* rows -> SQ8 */
  double assign_ms;             /* rectangular top-k kernel + its exact fallback */
  double fragment_ms;           /* tie key -> leader index, point ids */
  uint64_t rows;
  uint64_t fallback_rows;       /* rows recomputed by the exact sequential rule */
  uint32_t leaders;
  uint32_t fanout;
  uint32_t padded_dim;
} tessa_d0_profile;

TESSA_API int tessa_d0_last_profile(const tessa_ctx* ctx, tessa_d0_profile* out);

/* Device-pointer form: every array is a device pointer except leader_ids,
 * which may be either (it is read on the host to build the tie keys). */
TESSA_API int tessa_quantize_sq8_assign_d0(tessa_ctx* ctx, const tessa_d0_args* args, void* stream);
/* Host-pointer form: every array is a host pointer; the call uploads, runs
 * and downloads (the form the trait method binds). */
TESSA_API int tessa_quantize_sq8_assign_d0_host(tessa_ctx* ctx, const tessa_d0_args* args);

/* ------------------------------------------------------ candidate edges --- */

/* Largest sketch width / hash bit count (compute_hash asserts m_bits <= 16,
 * P/hash_prune.rs:2239-2241). */
#define TESSA_MAX_HASH_BITS 16

/* Per-point sketches for the HashPrune reducer: sketches[i*m + h] = the f32
 * sum over axes in order of x[i][a] * hyperplanes[h][a], one rounding per
 * multiply and per add -- fill_sketch_row (P/hash_prune.rs:2208-2232) as
 * compute_sketches_from_store calls it (:2155-2194).  The hyperplanes (m x dim,
 * from generate_hyperplanes, :2196-2206) are an input.  Device pointers. */
TESSA_API int tessa_sketch_rows(tessa_ctx* ctx, const float* x, uint64_t rows, uint32_t dim, const float* hyperplanes,
                                uint32_t m, float* sketches, void* stream);

/* Both personalised-residual hashes of every (row, rank) slot of a batch of
 * leaves, for the edge flush of flush_compact_topk_batch_into_edges
 * (P/leaf_build.rs:1749-1808): with i = point_ids[row], j = topk_ids[row*k +
 * rank], hash_fwd = compute_hash(sketch_i, sketch_j) and hash_rev =
 * compute_hash(sketch_j, sketch_i) (P/hash_prune.rs:2239-2251: bit b set iff
 * sketch_c[b] - sketch_p[b] >= 0).  Sketch rows are indexed by global point id
 * (the reference's SketchStore), sketch_width floats apart; slots whose id is
 * 0xffffffff get 0.  point_ids, topk_ids, sketches and the outputs are device
 * pointers.  leaf_starts / leaf_sizes (HOST arrays, leaf_count entries) give
 * the leaves as row ranges, each one CompactTopKBatch: the leaf's sketches are
 * then staged once in shared memory, and a candidate that is not a member of
 * its leaf is TESSA_ERR_BAD_TASK as in the reference (P/leaf_build.rs:
 * 1771-1777).  With leaf_count == 0 (or leaves too large to stage) every
 * candidate's sketch is read from the store directly, without that check. */
TESSA_API int tessa_edge_hashes(tessa_ctx* ctx, const uint32_t* point_ids, const uint32_t* topk_ids, uint64_t rows,
                                uint32_t k, const uint64_t* leaf_starts, const uint64_t* leaf_sizes,
                                uint64_t leaf_count, const float* sketches, uint64_t sketch_rows,
                                uint32_t sketch_width, uint32_t m_bits, uint16_t* hash_fwd, uint16_t* hash_rev,
                                void* stream);

/* Host-side edge expansion of a leaf batch in the reference's order
 * (P/leaf_build.rs:1749-1808): for each row, each rank with a valid id and a
 * finite distance, the edge (i -> j, hash_fwd, d) then (j -> i, hash_rev, d).
 * Host pointers; no device work.  With edge_p == NULL (or a capacity below the
 * count) only *edge_count is set; `threads` host threads (0 = 1). */
TESSA_API int tessa_expand_edges(const uint32_t* point_ids, const uint32_t* topk_ids, const float* topk_dists,
                                 const uint16_t* hash_fwd, const uint16_t* hash_rev, uint64_t rows, uint32_t k,
                                 uint32_t threads, uint32_t* edge_p, uint32_t* edge_c, uint16_t* edge_hash,
                                 float* edge_dist, uint64_t capacity, uint64_t* edge_count);

/* -------------------------------------------------------------- capture --- */

/* Membership digests of leaf tasks for the TESSA capture sampler: for leaf l
 * (rows leaf_starts[l] .. + leaf_sizes[l] of `ids`, HOST layout arrays) the
 * wrapping sum of mix(id) and the xor of rotl(mix(id), id & 63) over its
 * member ids, mix = the splitmix64 finaliser of id + 0x9e3779b97f4a7c15
 * (P/tessa_capture.rs:274-293, the digest every task hash covers).  With
 * global_ids non-NULL the member id is global_ids[ids[i]].  ids, global_ids
 * and the outputs (leaf_count u64 each) are device pointers. */
TESSA_API int tessa_membership_digests(tessa_ctx* ctx, const uint32_t* ids, const uint32_t* global_ids,
                                       const uint64_t* leaf_starts, const uint64_t* leaf_sizes, uint64_t leaf_count,
                                       uint64_t* out_sum, uint64_t* out_xor, void* stream);

/* ------------------------------------------------------- graph search --- */

/* Greedy search for recall runs (apps/search_shear_index/src/main.rs
 * search_one_with_stats :1007-1085, l2_distance :1639-1644): per query, the k
 * nearest ids found with list size l (l_eff = max(l, k + 1)) starting at
 * `start`, over a graph given as CSR (offsets[n + 1], neighbors); exact f32
 * squared L2 summed in axis order.  HOST pointers; `threads` host threads
 * (0 = 1).  Slots beyond the found results are 0xffffffff.  *comparisons
 * (optional) receives the distance evaluations. */
TESSA_API int tessa_graph_search(const float* data, uint64_t n, uint32_t dim, const uint64_t* offsets,
                                 const uint32_t* neighbors, uint32_t start, const float* queries, uint64_t nq,
                                 uint32_t k, uint32_t l, uint32_t threads, uint32_t* out_ids, uint64_t* comparisons);

/* ------------------------------------------------------- replay session --- */

/* TessaPreparedReplay (P/tessa_replay.rs:1052-1074) as host arrays. */
typedef struct tessa_prepared_replay {
  uint32_t dim;
  uint32_t padded_dim;
  uint64_t resident_rows;        /* = len(global_ids) */
  const uint32_t* global_ids;
  const float* vectors;          /* resident_rows x dim */
  const float* raw_norms;
  const int8_t* sq8_codes;       /* resident_rows x padded_dim */
  const float* sq8_scales;
  const float* sq8_norms;
  const uint32_t* assignment_members;
  uint64_t assignment_member_rows;
  const uint32_t* assignment_leaders;
  uint64_t assignment_leader_rows;
  const uint32_t* task_member_offsets;
  const uint32_t* task_member_counts;
  const uint32_t* task_leader_offsets;
  const uint32_t* task_leader_counts;
  const uint32_t* task_rh;
  const uint64_t* task_output_offsets;
  uint32_t task_count;
  uint64_t assignment_output_len;
  const uint32_t* leaf_members;
  uint64_t leaf_rows;
  const uint64_t* leaf_starts;
  const uint64_t* leaf_sizes;
  uint64_t leaf_count;
  uint32_t leaf_k;
} tessa_prepared_replay;

/* TessaReplayMode (P/tessa_replay.rs:18-86), same order and codes. */
#define TESSA_MODE_A0_FP32_SIMT 0u
#define TESSA_MODE_A1_TF32_WMMA 1u
#define TESSA_MODE_A2_SQ8_DP4A_BATCH1 2u
#define TESSA_MODE_A3_SQ8_WMMA_BATCH8 3u
#define TESSA_MODE_SQ8_DP4A_BATCH8 4u
#define TESSA_MODE_SQ8_WMMA_BATCH1 5u

/* ---------------------------------------------------- failure path --- */

/* Limit of every bounded device wait of the context's kernels (default 2 s;
 * 0 restores it; 10 ms .. 60 s).  A wait that runs out records
 * TESSA_DEVERR_TIMEOUT, every role of the kernel drains (waiting, under the
 * same limit, for its copies and MMAs in flight), tensor memory is freed and
 * the call returns TESSA_ERR_TIMEOUT -- as the reference's watchdog gives up
 * with a status instead of trapping (CB:5024-5025, CB:5883-5930). */
TESSA_API int tessa_set_wait_timeout_ns(tessa_ctx* ctx, uint64_t timeout_ns);

/* Self-test of that failure path (no counterpart in the reference): one CTA
 * waits, through the library's bounded wait, on a shared-memory barrier that
 * nothing arrives on, while a second warp waits with a much longer limit.  The
 * first wait gives up after timeout_ns (1 us .. 60 s) and raises the CTA's
 * abort flag, the second warp leaves at its next check, and the call returns
 * TESSA_ERR_TIMEOUT with *elapsed_ns (may be NULL) the kernel's own wait time.
 * The context stays usable.  No copy or MMA is in flight during the probe. */
TESSA_API int tessa_check_bounded_wait(tessa_ctx* ctx, uint64_t timeout_ns, uint64_t* elapsed_ns, void* stream);

/* ------------------------------------------------ subtree partition --- */

/* One batch of D1+ subtree tasks (GpuSubtreePartitionRequest, CB:1818-1826,
 * one per child run) for the recursive leader partition of the reference's
 * persistent kernel gpu_persistent_subtree_topk (CB:16336-17381).  Task t has
 * the resident rows task_members[task_offsets[t] .. + task_counts[t]),
 * ascending; inside a task rows are named by position (the reference's
 * subtree-local resident ids), which the leader sampler and the assignment tie
 * key hash.  Parameters are the persistent plan's (CB:1309-1340 with
 * PiPNNParams defaults, P/params.rs:3342-3368): leaf_max = max(256, c_max),
 * leaf_min 64, max_depth 10, max_leaders min(params.max_leaders, 128),
 * fanout_second 3 (root fanout, at most 4), root_depth = request.depth,
 * small_node_limit 4096, psamp_fraction 0.001; task_seeds as
 * gpu_queue_root_seed (CB:1597-1603).
 *
 * Result: leaves of at most leaf_max rows, written as resident ids into
 * leaf_rows (device) at leaf_starts[l] with leaf_sizes[l] rows from task
 * leaf_tasks[l] (host arrays).  Rows of a leaf ascend.  leaf_rows_capacity of
 * fanout_second * member_rows always suffices (the extent used may contain
 * gaps); leaf_capacity of the same bound too.  Leaves come in round order: all
 * leaves emitted by the nodes of one level, node by node, before the next.
 * The reference scatters rows into children with atomics (CB:15615-15626),
 * so its child order and deeper leaders vary from run to run; this call uses
 * the sequential order (rows ascending), which is deterministic. */
typedef struct tessa_subtree_args {
  const int8_t* codes;         /* device, resident_rows x padded_dim SQ8 codes */
  const float* scales;         /* device */
  const float* sq8_norms;      /* device */
  uint64_t resident_rows;
  uint32_t padded_dim;
  const uint32_t* task_members;  /* device */
  uint64_t member_rows;          /* entries of task_members */
  const uint64_t* task_offsets;  /* host, task_count */
  const uint32_t* task_counts;   /* host */
  const uint64_t* task_seeds;    /* host */
  uint32_t task_count;
  uint32_t leaf_max, leaf_min, max_depth, max_leaders, fanout_second, root_depth, small_node_limit;
  float psamp_fraction;
  uint32_t* leaf_rows;           /* device, leaf_rows_capacity entries */
  uint64_t leaf_rows_capacity;
  uint64_t* leaf_starts;         /* host, leaf_capacity entries */
  uint32_t* leaf_sizes;          /* host */
  uint32_t* leaf_tasks;          /* host, may be NULL */
  uint64_t leaf_capacity;
  /* Optional (may be NULL): device output of leaf_rows_capacity x padded_dim
   * bytes; row p receives the codes of leaf_rows[p] (zeros where the arena
   * holds no row) -- the leaf-ordered codes tessa_leaf_topk_sq8 takes as
   * leaf_ordered_codes.  Each round's leaves are copied while the host
   * decides the next round. */
  int8_t* leaf_codes;
} tessa_subtree_args;

typedef struct tessa_subtree_result {
  uint64_t leaf_count;
  uint64_t leaf_rows_used;       /* extent of leaf_rows written */
  uint32_t rounds;               /* levels (plus retry rounds) */
  uint32_t large_assignments;    /* node assignments on the tensor cores */
  uint32_t retries;              /* large-node leader resamples (CB:15416-15478) */
  uint32_t balanced;             /* balanced even/odd fallbacks (CB:15480-15504) */
  uint32_t small_nodes;          /* subtree roots split on the small path */
  uint32_t kernel_launches;      /* kernels this call launched */
  float assign_ms;               /* device time of the large-node assignment phases (all rounds) */
  float scatter_ms;              /* device time of the scatter phases */
  float small_ms;                /* device time of the small-node path */
  float wall_ms;                 /* host wall time of the call */
  float host_prep_ms;            /* host time building each round's node tables */
  float host_decide_ms;          /* host time deciding splits and allocating */
  float sync_wait_ms;            /* host time waiting on the stream */
} tessa_subtree_result;

/* The partition of one batch of subtree tasks (synchronous on `stream`).
 * Replaces the partition workers of gpu_persistent_subtree_topk behind
 * PiPNNComputeBackend::process_quantized_subtree_l2_compact_topk (CB:3693-3884);
 * the leaves then go to tessa_leaf_topk_sq8.  Entries of leaf_rows that belong
 * to no leaf (unused reservations of the small-node path) hold 0xffffffff. */
TESSA_API int tessa_subtree_partition(tessa_ctx* ctx, const tessa_subtree_args* args, tessa_subtree_result* result,
                                      void* stream);

/* Subtree submissions: submit_owned_quantized_subtree_l2_compact_topk
 * (CB:3693-3884) with the persistent async D2H ring
 * (P/persistent_async_d2h.rs:4-80, two slots).  A submission partitions a
 * batch of subtree tasks (as tessa_subtree_partition; the output fields of
 * `partition` are ignored -- the slot owns the leaf arena), evaluates every
 * leaf (as tessa_leaf_topk_sq8 with `global_ids` and `k`), and copies the
 * CompactTopKBatch (P/leaf_build.rs:271-290) -- the global id of every leaf
 * row, its k ids and distances -- into the slot's pinned host memory.
 *
 * tessa_subtree_submit copies the request's host arrays, records `stream`
 * (the submission starts after the work queued on it so far) and returns at
 * once with a ticket; the work runs on a private context of the same device
 * (its own stream and scratch), in submission order.  The device inputs
 * (codes, scales, norms, task_members, global_ids) must stay valid until the
 * ticket is polled.  With both slots leased it returns TESSA_ERR_AGAIN.
 * tessa_subtree_poll fills `view` once the batch is on the host (wait = 0:
 * TESSA_ERR_AGAIN while it runs; wait != 0: blocks); a failed submission
 * returns its error and frees its slot.  The view's arrays stay valid until
 * tessa_subtree_release(ticket), which frees the slot.  Leaf rows that belong
 * to no leaf have point id 0xffffffff and k empty slots. */
typedef struct tessa_subtree_request {
  tessa_subtree_args partition;
  const uint32_t* global_ids;    /* device, resident_rows: local id -> point id */
  uint32_t k;                    /* 1 .. TESSA_MAX_LEAF_K */
} tessa_subtree_request;

typedef struct tessa_compact_view {
  uint64_t ticket;
  uint64_t rows;                 /* leaf rows of the batch */
  uint32_t k;
  uint64_t leaf_count;
  const uint64_t* leaf_starts;   /* host, leaf_count: first row of each leaf */
  const uint32_t* leaf_sizes;    /* host, leaf_count */
  const uint32_t* leaf_tasks;    /* host, leaf_count: task index in the request */
  const uint32_t* point_ids;     /* pinned host, rows */
  const uint32_t* topk_ids;      /* pinned host, rows * k (0xffffffff: none) */
  const float* topk_dists;       /* pinned host, rows * k */
  tessa_subtree_result partition;
  uint64_t fallback_rows;        /* leaf rows recomputed by the exact sequential kernel */
} tessa_compact_view;

TESSA_API int tessa_subtree_submit(tessa_ctx* ctx, const tessa_subtree_request* request, uint64_t* ticket,
                                   void* stream);
TESSA_API int tessa_subtree_poll(tessa_ctx* ctx, uint64_t ticket, int wait, tessa_compact_view* view);
TESSA_API int tessa_subtree_release(tessa_ctx* ctx, uint64_t ticket);

/* ---------------------------------------------------- host reduction --- */

/* One candidate edge of a reservoir: the target point, the SQ8 distance and
 * the personalised-residual hash (hash_prune.rs:2239-2251). */
typedef struct tessa_edge {
  uint32_t target;
  float dist;
  uint16_t hash;
  uint16_t reserved;
} tessa_edge;

/* Candidate records of a leaf batch grouped by reservoir on the device: the
 * edges of flush_compact_topk_batch_into_edges (P/leaf_build.rs:1749-1808; for
 * row i and rank r with id j != 0xffffffff and a finite distance d,
 * (point_ids[i] -> j, hash_fwd, d) and (j -> point_ids[i], hash_rev, d)) laid
 * out so that point p's edges are edges[offsets[p] .. offsets[p+1]), ascending
 * by target.  An edge that repeats another exactly (same source, target, hash
 * and distance -- overlapping leaves produce every edge many times) is kept
 * once: a reservoir ignores a repeated candidate, so the reduction's result is
 * unchanged.  All pointers are device pointers; offsets has num_points + 1
 * entries, edges edge_capacity >= 2 * rows * k; 2 * rows * k must be below
 * 2^32.  Ids at or above num_points are TESSA_ERR_BAD_ROW.  Synchronous on
 * `stream`. */
TESSA_API int tessa_group_edges(tessa_ctx* ctx, const uint32_t* point_ids, const uint32_t* topk_ids,
                                const float* topk_dists, const uint16_t* hash_fwd, const uint16_t* hash_rev,
                                uint64_t rows, uint32_t k, uint64_t num_points, uint64_t* offsets, tessa_edge* edges,
                                uint64_t edge_capacity, void* stream);

/* HashPrune reservoirs on the host (HashPruneReservoir,
 * P/hash_prune.rs:269-1452), the CPU-side reduction SHEAR feeds its leaf
 * candidate records into.  One reservoir of at most l_max slots per point
 * (l_max <= 255; PiPNNParams l_max 64); `threads` host threads (0 = 1).
 * Host pointers throughout.  A reducer is not thread-safe. */
typedef struct tessa_reducer tessa_reducer;
TESSA_API int tessa_reducer_create(uint64_t num_points, uint32_t l_max, uint32_t threads, tessa_reducer** out);
/* One CompactTopKBatch (P/leaf_build.rs:271-290) flushed as
 * flush_compact_topk_batch_into_edges forms its edges (P/leaf_build.rs:
 * 1749-1808): for row i and rank r with id j != 0xffffffff and a finite
 * distance d, (point_ids[i] -> j, hash_fwd, d) then (j -> point_ids[i],
 * hash_rev, d), each inserted with insert_inner (P/hash_prune.rs:1326-1452).
 * Ids at or above num_points are TESSA_ERR_BAD_ROW. */
TESSA_API int tessa_reducer_add(tessa_reducer* reducer, const uint32_t* point_ids, const uint32_t* topk_ids,
                                const float* topk_dists, const uint16_t* hash_fwd, const uint16_t* hash_rev,
                                uint64_t rows, uint32_t k);
/* Edges already grouped by reservoir (host copies of tessa_group_edges'
 * outputs: offsets has num_points + 1 entries): each reservoir takes its
 * group; the result equals tessa_reducer_add on the same records. */
TESSA_API int tessa_reducer_add_grouped(tessa_reducer* reducer, const uint64_t* offsets, const tessa_edge* edges);
/* Final neighbour lists, each point's slot targets in hash order (the
 * resident emit with backfill off, P/mod.rs:2437-2478), as CSR: offsets
 * (num_points + 1 entries) and neighbors (capacity entries; NULL to size). */
TESSA_API int tessa_reducer_finish(const tessa_reducer* reducer, uint64_t* offsets, uint32_t* neighbors,
                                   uint64_t capacity, uint64_t* count);
/* Edges inserted so far (forward and reverse). */
TESSA_API int tessa_reducer_edges(const tessa_reducer* reducer, uint64_t* edges);
TESSA_API void tessa_reducer_destroy(tessa_reducer* reducer);

/* HashPrune reservoirs built on the device.  The result equals the host
 * reducer above (and the reference's sequence of insert_inner calls,
 * P/hash_prune.rs:1326-1452) on the same edges: each source's slots are the
 * l_max best, in the total order (distance via total_cmp, target, hash) of
 * P/hash_prune.rs:2094-2130, of the per-hash minima of its edges, written in
 * hash order.  Outputs (device): out_offsets (num_points + 1 entries) and the
 * slots as neighbour ids (out_neighbors) and/or full slots (out_slots, which
 * can be fed back as grouped input); either may be NULL.  slot_capacity >=
 * min(edges, num_points * l_max) always suffices; *slot_count (host) gets the
 * slot total, and a capacity below it is TESSA_ERR_INVALID_ARG after the
 * offsets are written.  l_max in 1..255.  Synchronous on `stream`.
 *
 * tessa_reduce_records takes leaf records as tessa_reducer_add does (device
 * pointers; ids at or above num_points are TESSA_ERR_BAD_ROW; 2 * rows * k
 * below 2^32).  tessa_reduce_grouped takes `groups` pieces of edges grouped by
 * source over points 0 .. num_points-1 -- piece g: group_offsets[g] (device,
 * num_points + 1 entries, not necessarily starting at 0) and group_edges[g]
 * (device, group_edge_counts[g] edges from group_offsets[g][0] on); the
 * pointer arrays and counts are host arrays -- such as tessa_group_edges'
 * output or other reservoirs' out_slots.  Edges with a non-finite distance are
 * skipped; the sum of the counts must be below 2^32. */
TESSA_API int tessa_reduce_records(tessa_ctx* ctx, const uint32_t* point_ids, const uint32_t* topk_ids,
                                   const float* topk_dists, const uint16_t* hash_fwd, const uint16_t* hash_rev,
                                   uint64_t rows, uint32_t k, uint64_t num_points, uint32_t l_max,
                                   uint64_t* out_offsets, uint32_t* out_neighbors, tessa_edge* out_slots,
                                   uint64_t slot_capacity, uint64_t* slot_count, void* stream);
TESSA_API int tessa_reduce_grouped(tessa_ctx* ctx, uint32_t groups, const uint64_t* const* group_offsets,
                                   const tessa_edge* const* group_edges, const uint64_t* group_edge_counts,
                                   uint64_t num_points, uint32_t l_max, uint64_t* out_offsets,
                                   uint32_t* out_neighbors, tessa_edge* out_slots, uint64_t slot_capacity,
                                   uint64_t* slot_count, void* stream);

/* TessaCudaModeResult (P/tessa_replay.rs:190-200); caller-owned host buffers
 * of assignment_output_len and leaf_rows*leaf_k entries.  leaf_* may be NULL
 * for modes that replay no leaf tasks. */
typedef struct tessa_mode_result {
  double assignment_event_ms;
  double leaf_event_ms;          /* < 0 when the mode replays no leaf tasks */
  double total_event_ms;
  uint32_t* assignment_ids;
  float* assignment_dists;
  uint32_t* leaf_ids;
  float* leaf_dists;
  uint64_t device_error_bits;    /* OR of kernel error words (0 = clean) */
} tessa_mode_result;

/* TessaCudaReplaySession::new (CB:34649-34839): uploads the prepared replay
 * once. */
TESSA_API int tessa_replay_session_create(int device, const tessa_prepared_replay* prepared,
                                tessa_replay_session** out);
/* TessaCudaReplaySession::run_mode (CB:34841-34969): clears outputs, runs the
 * assignment and (for modes A0-A3) leaf operators between CUDA events,
 * downloads the results and applies the safety gate. */
TESSA_API int tessa_replay_run_mode(tessa_replay_session* session, uint32_t mode, tessa_mode_result* result);
TESSA_API void tessa_replay_session_destroy(tessa_replay_session* session);

#ifdef __cplusplus
}
#endif

#endif /* TESSA_SM100_H */
