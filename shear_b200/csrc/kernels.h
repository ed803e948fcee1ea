// Host-visible launch descriptors and launchers of the TESSA sm_100a kernels
// (defined in leaf_sq8.cu, quantize_sq8.cu and assign.cu, called by capi.cu).
#pragma once
#include <stdint.h>
#include <cuda_runtime.h>

#include "../../include/tessa_sm100.h"

namespace tessa {

struct LeafLaunch {
  const int8_t* leaf_codes;   // leaf-ordered codes (row p = member p)
  uint64_t leaf_rows;
  uint32_t padded_dim;
  const float* scales;        // by local id
  const float* norms;
  const uint32_t* global_ids;
  const uint32_t* members;    // leaf-ordered local ids
  const uint64_t* d_leaf_starts;
  const uint32_t* d_leaf_sizes;
  const uint2* d_tiles;       // (leaf, first row) per 128-row tile
  uint32_t num_tiles;
  uint32_t k;
  uint32_t* out_ids;
  float* out_dists;
  uint32_t* d_err;
  uint32_t* d_fb_count;       // scratch: number of rows handed to the exact fallback
  uint2* d_fb_list;           // scratch: (leaf, row) of those rows, fb_capacity entries
  uint32_t fb_capacity;
  uint64_t resident_rows;     // bound for member ids
  uint64_t timeout_ns;
  int sm_count;
  // Column-split kernel (padded_dim <= 1024): per-row zone dump for rows
  // [dump_row0, dump_row0 + dump_rows) of the leaf-ordered row space,
  // leaf_dump_bytes(dump_rows, k) bytes at d_dump.  Null: the four-warp kernel.
  void* d_dump = nullptr;
  uint64_t dump_row0 = 0;
  uint64_t dump_rows = 0;
  // Column-split kernel on CTA pairs (two SMs share each B chunk): 256-row
  // tile pairs (leaf, first row); null or zero: one CTA per tile.
  const uint2* d_pairs = nullptr;
  uint32_t num_pairs = 0;
};

// Column-split leaf kernel: shared-memory plan (false: not supported for this
// padded_dim / k) and the dump scratch it needs for `rows` leaf rows.
bool leaf_split_plan(uint32_t padded_dim, uint32_t k, uint32_t* ring, uint32_t* log_cap);
uint64_t leaf_dump_bytes(uint64_t rows, uint32_t k);
uint64_t leaf_dump_m_offset(uint64_t rows, uint32_t k);
uint32_t leaf_dump_entries(uint32_t k);

// Largest leaf the leaf kernel accepts (a validated cap above the reference's
// leaf sizes).
constexpr uint64_t kMaxLeafRows = 65535;

// Rectangular form of the leaf kernel: each row of a row matrix against every
// row (column) of a second matrix, per-row bounded top-k under the same
// eps/id rule, the column's tie key as the id (global-D0 assignment).
struct RectLaunch {
  const int8_t* row_codes;    // rows x padded_dim
  uint64_t rows;
  uint32_t padded_dim;
  const float* row_scales;
  const float* row_norms;
  const int8_t* col_codes;    // cols x padded_dim
  uint32_t cols;
  const float* col_scales;
  const float* col_norms;
  const uint32_t* col_keys;   // distinct tie keys; output ids are these keys
  uint32_t k;
  uint32_t* out_keys;         // rows x k
  float* out_dists;           // rows x k
  uint32_t* d_err;
  uint32_t* d_fb_count;
  uint2* d_fb_list;           // capacity fb_capacity (>= rows suffices)
  uint32_t fb_capacity;
  uint64_t timeout_ns;
  int sm_count;
};

// Row tiles are indexed in 32 bits.
constexpr uint64_t kMaxRectRows = 0xffffff00ull;

int launch_leaf_topk_sq8(const LeafLaunch& L, cudaStream_t stream);
int launch_rect_topk_sq8(const RectLaunch& R, cudaStream_t stream);
int launch_d0_fragments(const uint32_t* keys, const uint32_t* key_to_leader, const uint32_t* global_ids, uint64_t rows,
                        uint32_t fanout, uint32_t leaders, uint32_t* child_ids, uint32_t* point_ids, uint32_t* d_err,
                        int sm_count, cudaStream_t stream);
int launch_sketch_rows(const float* x, uint64_t rows, uint32_t dim, const float* planes, uint32_t m, float* out,
                       int sm_count, cudaStream_t stream);
int launch_edge_hashes(const uint32_t* point_ids, const uint32_t* topk_ids, uint64_t rows, uint32_t k,
                       const float* sketches, uint64_t sketch_rows, uint32_t width, uint32_t m_bits,
                       uint16_t* hash_fwd, uint16_t* hash_rev, uint32_t* d_err, int sm_count, cudaStream_t stream);
// Per-leaf hashes (leaf layout on the device); TESSA_ERR_UNSUPPORTED if the
// largest leaf's sketches and id table exceed kLeafEdgeSmemMax.
constexpr uint32_t kLeafEdgeSmemMax = 200u * 1024u;
uint32_t leaf_edge_smem(uint32_t max_rows, uint32_t m_bits, uint32_t* log2cap);
int launch_leaf_edge_hashes(const uint32_t* point_ids, const uint32_t* topk_ids, const uint64_t* d_leaf_starts,
                            const uint32_t* d_leaf_sizes, uint32_t leaf_count, uint32_t max_rows, uint32_t k,
                            const float* sketches, uint64_t sketch_rows, uint32_t width, uint32_t m_bits,
                            uint16_t* hash_fwd, uint16_t* hash_rev, uint32_t* d_err, int sm_count,
                            cudaStream_t stream);
// Returns the edge count; writes the edges only if out_p is non-null and the
// count fits `capacity`.
uint64_t expand_edges_host(const uint32_t* point_ids, const uint32_t* topk_ids, const float* topk_dists,
                           const uint16_t* hash_fwd, const uint16_t* hash_rev, uint64_t rows, uint32_t k,
                           uint32_t* out_p, uint32_t* out_c, uint16_t* out_hash, float* out_dist, uint64_t capacity,
                           uint32_t threads);
int launch_membership_digests(const uint32_t* ids, const uint32_t* global_ids, const uint64_t* d_leaf_starts,
                              const uint64_t* d_leaf_sizes, uint32_t leaf_count, uint64_t* out_sum,
                              uint64_t* out_xor, int sm_count, cudaStream_t stream);
// Greedy search of nq queries over a CSR graph (host threads); returns the
// number of distance evaluations.
uint64_t graph_search_host(const float* data, uint64_t n, uint32_t dim, const uint64_t* offsets,
                           const uint32_t* neighbors, uint32_t start, const float* queries, uint64_t nq, uint32_t k,
                           uint32_t l, uint32_t threads, uint32_t* out_ids);
int launch_gather_rows(const int8_t* src, const uint32_t* members, uint64_t rows, uint32_t row_bytes,
                       uint64_t resident_rows, int8_t* dst, int sm_count, cudaStream_t stream);
int leaf_num_bstages(uint32_t padded_dim);
int launch_quantize_sq8(const float* x, uint64_t rows, uint32_t dim, uint32_t padded, uint32_t bits, int8_t* codes,
                        float* scales, float* norms, uint32_t* d_err, cudaStream_t stream);

namespace assign {
struct Params {
  const float* x;
  const float* raw_norms;
  const int8_t* codes;
  const float* scales;
  const float* sq8_norms;
  const uint32_t* global_ids;
  uint64_t resident_rows;
  uint32_t dim;
  uint32_t padded_dim;
  const uint32_t* members;
  const uint32_t* leaders;
  const uint32_t* t_moff;
  const uint32_t* t_mcnt;
  const uint32_t* t_loff;
  const uint32_t* t_lcnt;
  const uint32_t* t_rh;
  const uint64_t* t_out;
  const uint2* work;          // (task, first row) per 128-row work item
  uint32_t num_work;
  uint32_t fused;             // SQ8 distance as one FFMA (1) or one rounding per op (0)
  uint32_t* out_ids;
  float* out_dists;
  uint32_t* err_word;
  uint64_t timeout_ns = 2000000000ull;  // bound of every wait in the tensor-core kernel
  // Slot mode (the subtree partition, SQ8 tensor-core kernel only): when
  // out_slots is set, each row keeps a list of t_rh[task] slots (not four),
  // the insertion's tie keys hash member_tie / leader_tie (parallel to
  // members / leaders: subtree-local ids) instead of the resident rows, and
  // the result is the leader slot index per rank in out_slots (out_dists is
  // written when non-null, out_ids is not used).
  const uint32_t* member_tie = nullptr;
  const uint32_t* leader_tie = nullptr;
  uint32_t* out_slots = nullptr;
};
}  // namespace assign

// SQ8 sources go to the tensor-core kernel (assign_tc.cu) when every task has
// at most 128 leaders, to the SIMT kernel otherwise; FP32 sources to the SIMT
// kernel.
int launch_assign(const assign::Params& prm, bool sq8, uint32_t max_leaders, int sm_count, cudaStream_t stream);
int launch_assign_sq8_tc(const assign::Params& prm, uint32_t max_leaders, int sm_count, cudaStream_t stream);

// Recursive subtree partition (subtree.cu); scratch owned by the context.
struct SubtreeState;
SubtreeState* subtree_state_new();
void subtree_state_free(SubtreeState* s);
struct SubtreeStats {
  uint64_t leaf_count, leaf_rows_used;
  uint32_t rounds, large_assignments, retries, balanced, small_nodes, launches;
  float assign_ms, scatter_ms, small_ms, wall_ms;
  float host_prep_ms, host_decide_ms, sync_wait_ms;  // host time: round set-up, decisions, stream waits
};
int subtree_partition(SubtreeState* s, const tessa_subtree_args& a, SubtreeStats* stats, uint32_t* d_err,
                      int sm_count, uint64_t timeout_ns, cudaStream_t stream);

// Candidate records grouped by reservoir (records.cu).
struct GroupEdgesCall {
  const uint32_t* point_ids;
  const uint32_t* topk_ids;
  const float* topk_dists;
  const uint16_t* hash_fwd;
  const uint16_t* hash_rev;
  uint64_t rows;
  uint32_t k;
  uint64_t num_points;
  uint64_t* offsets;      // num_points + 1
  tessa_edge* edges;      // capacity >= 2 * rows * k
  void* temp;             // group_edges_scratch_bytes(2 * rows * k, num_points)
  size_t temp_bytes;
  uint32_t* d_err;
  int sm_count;
};
int group_edges(const GroupEdgesCall& g, cudaStream_t stream);
size_t group_edges_scratch_bytes(uint64_t edges, uint64_t num_points);

// Device HashPrune reservoirs (reservoirs.cu): leaf records (groups == 0) or
// edges grouped by source in `groups` CSR pieces -> each source's l_max best
// per-hash minima in hash order.
struct ReservoirCall {
  const uint32_t* point_ids;
  const uint32_t* topk_ids;
  const float* topk_dists;
  const uint16_t* hash_fwd;
  const uint16_t* hash_rev;
  uint64_t rows;
  uint32_t k;
  uint32_t groups;
  const uint64_t* const* group_offsets;  // host array of device pointers
  const tessa_edge* const* group_edges;  // host array of device pointers
  const uint64_t* group_counts;          // host array
  uint64_t edges;                        // 2 * rows * k, or the sum of group_counts
  uint64_t num_points;
  uint32_t l_max;
  uint64_t* out_offsets;
  uint32_t* out_neighbors;
  tessa_edge* out_slots;
  uint64_t capacity;
  void* temp;  // reservoir_scratch_bytes(edges, num_points)
  size_t temp_bytes;
  uint32_t* d_err;
  int sm_count;
};
int reduce_reservoirs(const ReservoirCall& r, cudaStream_t stream);
// Subtree submissions (submit.cu): a two-slot ring run by a worker thread on a
// private context of the same device.
struct SubmitRing;
int submit_ring_create(int device, SubmitRing** out);
void submit_ring_destroy(SubmitRing* ring);
int submit_ring_submit(SubmitRing* ring, const tessa_subtree_request* req, uint64_t* ticket, cudaStream_t caller);
int submit_ring_poll(SubmitRing* ring, uint64_t ticket, int wait, tessa_compact_view* view);
int submit_ring_release(SubmitRing* ring, uint64_t ticket);
size_t reservoir_scratch_bytes(uint64_t edges, uint64_t num_points);

// Records `code` and `message` as the calling thread's last error (returned by
// tessa_last_error_message); returns `code`.
int set_last_error(int code, const char* message);

}  // namespace tessa
