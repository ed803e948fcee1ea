/*
 * tessa_oracle.c -- CPU restatement of SHEAR's TESSA hot path, used ONLY as a
 * test/benchmark checker.  Nothing in the shipped library links or calls this
 * file: tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load it
 * through ctypes to check (or time) the CUDA path.
 *
 * Every function restates one piece of the reference (wbh1765091327/SHEAR,
 * Rust + NVRTC CUDA strings).  Citations are relative to the reference project
 * root; CB = shear-core/src/algorithm/pipnn/compute_backend.rs,
 * P  = shear-core/src/algorithm/pipnn/.
 *
 * Floating point: compiled with -ffp-contract=off so that every a*b and a+b is
 * one IEEE-754 binary32 rounding, as the reference's __fmul_rn/__fadd_rn and
 * Rust's non-contracting f32 arithmetic are.  Where the reference leaves
 * contraction to nvcc (SQ8 assignment distance, CB:14676-14678), both the
 * contracted (fmaf) and the uncontracted forms are provided.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <float.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORACLE_OK 0
#define ORACLE_ERR_ARG (-1)
#define ORACLE_ERR_NONFINITE (-2)
#define ORACLE_ERR_RANGE (-3)

#define TIE_EPS 2.0e-5f           /* P/mod.rs:74 STABLE_DISTANCE_TIE_EPS, CB:8077 */
#define EMPTY_DIST 3.402823466e+38F /* CB:9506 initial slot distance */
#define EMPTY_ID 0xffffffffu        /* CB:9507 initial slot id */
#define MAX_K 32u                   /* CB:4890 GPU_PERSISTENT_LEAF_DCO_MAX_SURVIVORS */

/* ---------------------------------------------------------------- SQ8 --- */

/* P/dco_sq_int8.rs:1216-1224 sq_int8_padded_dim */
uint32_t oracle_padded_dim(uint32_t dim, uint32_t k_align) {
    if (dim == 0) return 0;
    if (k_align == 0) k_align = 1;
    return ((dim + k_align - 1) / k_align) * k_align;
}

/*
 * P/dco_sq_int8.rs:1331-1375 quantize_sq_int8_matrix_with_bits and
 * :1431-1466 quantize_sq_int8_row_with_max_code.
 * max_code = 2^(bits-1)-1 (:1325-1329); norm = sequential f32 sum of x*x;
 * scale = max|x| / max_code (1.0 for an all-zero row);
 * code = clamp(round_half_away(x / scale), -max_code, max_code); zero padding.
 * Returns padded_dim, or a negative error.
 */
int64_t oracle_quantize_sq8(const float* x, uint64_t rows, uint32_t dim, uint32_t k_align,
                            uint32_t bits, int8_t* codes, float* scales, float* norms) {
    if (bits < 2 || bits > 8) return ORACLE_ERR_ARG;          /* :1316-1323 */
    uint32_t padded = oracle_padded_dim(dim, k_align);
    if (padded == 0) return ORACLE_ERR_ARG;
    float max_code = (float)((1u << (bits - 1)) - 1u);
    int bad = 0;
#pragma omp parallel for schedule(static) reduction(| : bad)
    for (int64_t row = 0; row < (int64_t)rows; ++row) {
        const float* in = x + (uint64_t)row * dim;
        int8_t* out = codes + (uint64_t)row * padded;
        memset(out, 0, padded);
        float max_abs = 0.0f, norm = 0.0f;
        for (uint32_t a = 0; a < dim; ++a) {
            float v = in[a];
            if (!isfinite(v)) { bad = 1; break; }
            float av = fabsf(v);
            max_abs = max_abs > av ? max_abs : av;
            norm = norm + v * v;
        }
        if (max_abs == 0.0f) {
            scales[row] = 1.0f;
            norms[row] = norm;
            continue;
        }
        float scale = max_abs / max_code;
        for (uint32_t a = 0; a < dim; ++a) {
            float c = roundf(in[a] / scale);
            if (c < -max_code) c = -max_code;
            if (c > max_code) c = max_code;
            out[a] = (int8_t)c;
        }
        scales[row] = scale;
        norms[row] = norm;
    }
    return bad ? ORACLE_ERR_NONFINITE : (int64_t)padded;
}

/* P/tessa_replay.rs:1287-1290: raw norms, sequential f32 sum of x*x. */
void oracle_raw_norms(const float* x, uint64_t rows, uint32_t dim, float* norms) {
#pragma omp parallel for schedule(static)
    for (int64_t row = 0; row < (int64_t)rows; ++row) {
        const float* in = x + (uint64_t)row * dim;
        float s = 0.0f;
        for (uint32_t a = 0; a < dim; ++a) s = s + in[a] * in[a];
        norms[row] = s;
    }
}

/* P/dco_sq_int8.rs:2685-2690 sq_int8_dot_scalar_unchecked (exact int32). */
int32_t oracle_sq8_dot(const int8_t* a, const int8_t* b, uint32_t padded_dim) {
    int32_t s = 0;
    for (uint32_t i = 0; i < padded_dim; ++i) s += (int32_t)a[i] * (int32_t)b[i];
    return s;
}

/*
 * CB:8987-9002 gpu_persistent_sq_int8_l2_from_dot:
 *   dist = rn(rn(n_i + n_j) + rn(-2 * rn(rn(s_i * s_j) * (float)dot))), clamp <= 0 to 0.
 * Equal to P/dco_sq_int8.rs:2950-2965 sq_int8_approx_l2 because 2* is exact.
 */
float oracle_sq8_l2_from_dot(int32_t dot, float row_scale, float row_norm, float col_scale,
                             float col_norm) {
    float ss = row_scale * col_scale;
    float sd = ss * (float)dot;
    float m2 = -2.0f * sd;
    float nn = row_norm + col_norm;
    float dist = nn + m2;
    if (dist <= 0.0f) dist = 0.0f;
    return dist;
}

/* ------------------------------------------------------------ leaf top-k --- */

/* CB:7229-7259 / 8068-8104 stable eps-id order ("better"). */
static inline int better(float d, uint32_t id, float od, uint32_t oid) {
    float delta = d - od;
    return (fabsf(delta) <= TIE_EPS) ? (id < oid) : (d < od);
}

/*
 * CB:7229-7259 gpu_persistent_insert_topk_candidate_fp32: reject unless better
 * than the last slot, then shift up while better than the previous slot.
 */
static inline void insert_topk(float d, uint32_t id, uint32_t k, float* bd, uint32_t* bi) {
    if (!better(d, id, bd[k - 1], bi[k - 1])) return;
    uint32_t pos = k - 1;
    while (pos > 0 && better(d, id, bd[pos - 1], bi[pos - 1])) {
        bd[pos] = bd[pos - 1];
        bi[pos] = bi[pos - 1];
        --pos;
    }
    bd[pos] = d;
    bi[pos] = id;
}

/*
 * Exact per-row leaf result (CB:9569-9650 scalar executor, CB:10046-10096 WMMA
 * consumer): columns in ascending member position over [col_begin, col_end),
 * skipping the row's own local id, distances per oracle_sq8_l2_from_dot,
 * inserted into a list of `slots` entries initialised to (FLT_MAX, 0xffffffff).
 * Output ids are the columns' global ids.
 */
static void leaf_row_partial(const int8_t* codes, const float* scales, const float* norms,
                             const uint32_t* global_ids, uint32_t padded_dim,
                             const uint32_t* members, uint32_t local_i, uint64_t col_begin,
                             uint64_t col_end, uint32_t slots, float* bd, uint32_t* bi) {
    for (uint32_t s = 0; s < slots; ++s) { bd[s] = EMPTY_DIST; bi[s] = EMPTY_ID; }
    if (slots == 0) return;
    const int8_t* rc = codes + (uint64_t)local_i * padded_dim;
    float rs = scales[local_i], rn = norms[local_i];
    for (uint64_t c = col_begin; c < col_end; ++c) {
        uint32_t local_j = members[c];
        if (local_j == local_i) continue;
        int32_t dot = oracle_sq8_dot(rc, codes + (uint64_t)local_j * padded_dim, padded_dim);
        float dist = oracle_sq8_l2_from_dot(dot, rs, rn, scales[local_j], norms[local_j]);
        insert_topk(dist, global_ids[local_j], slots, bd, bi);
    }
}

/*
 * Leaf top-k over a batch of leaves (the replay contract of
 * P/tessa_replay.rs:1337-1388 and CB:35189-35230):
 *   leaf l has members leaf_members[off_l .. off_l + cnt_l) (local row ids);
 *   its output row r is written at (off_l + r) * k.
 * col_task_width == 0: one sequential pass over all columns (the reference's
 *   path for every leaf of <= 512 rows, and the canonical order here).
 * col_task_width  > 0: the reference's staged replay path for leaves of more
 *   than 512 rows (CB:35199-35203): per column task of col_task_width columns a
 *   partial list is built (survivor limit min(k, task candidates),
 *   CB:9484-9497), then merged into the output row slot by slot
 *   (CB:7261-7309), tasks taken in ascending order.
 */
int oracle_leaf_topk_sq8(const int8_t* codes, const float* scales, const float* norms,
                         const uint32_t* global_ids, uint64_t resident_rows, uint32_t padded_dim,
                         const uint32_t* leaf_members, const uint64_t* leaf_offsets,
                         const uint64_t* leaf_counts, uint64_t leaf_count, uint32_t k,
                         uint32_t col_task_width, uint32_t staged_min_rows, uint32_t* out_ids,
                         float* out_dists) {
    if (k == 0 || k > MAX_K) return ORACLE_ERR_ARG;
    int bad = 0;
    for (uint64_t l = 0; l < leaf_count; ++l) {
        for (uint64_t r = 0; r < leaf_counts[l]; ++r)
            if (leaf_members[leaf_offsets[l] + r] >= resident_rows) bad = 1;
    }
    if (bad) return ORACLE_ERR_RANGE;
#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t l = 0; l < (int64_t)leaf_count; ++l) {
        const uint32_t* members = leaf_members + leaf_offsets[l];
        uint64_t cnt = leaf_counts[l];
        int staged = col_task_width > 0 && cnt > staged_min_rows;
        for (uint64_t r = 0; r < cnt; ++r) {
            float bd[MAX_K], pd[MAX_K];
            uint32_t bi[MAX_K], pi[MAX_K];
            uint32_t li = members[r];
            uint64_t out = (leaf_offsets[l] + r) * k;
            if (!staged) {
                uint64_t cand = cnt > 0 ? cnt - 1 : 0;
                uint32_t slots = cand < k ? (uint32_t)cand : k;
                leaf_row_partial(codes, scales, norms, global_ids, padded_dim, members, li, 0,
                                 cnt, slots, bd, bi);
                for (uint32_t s = slots; s < k; ++s) { bd[s] = EMPTY_DIST; bi[s] = EMPTY_ID; }
            } else {
                for (uint32_t s = 0; s < k; ++s) { bd[s] = EMPTY_DIST; bi[s] = EMPTY_ID; }
                for (uint64_t base = 0; base < cnt; base += col_task_width) {
                    uint64_t end = base + col_task_width < cnt ? base + col_task_width : cnt;
                    uint64_t cand = end - base;
                    if (r >= base && r < end && cand > 0) cand -= 1;
                    uint32_t slots = cand < k ? (uint32_t)cand : k;
                    leaf_row_partial(codes, scales, norms, global_ids, padded_dim, members, li,
                                     base, end, slots, pd, pi);
                    for (uint32_t s = 0; s < slots; ++s)
                        if (pi[s] != EMPTY_ID && isfinite(pd[s])) insert_topk(pd[s], pi[s], k, bd, bi);
                }
            }
            for (uint32_t s = 0; s < k; ++s) { out_ids[out + s] = bi[s]; out_dists[out + s] = bd[s]; }
        }
    }
    return ORACLE_OK;
}

/* ------------------------------------------------------ global D0 --- */

/*
 * P/dco_sq_int8.rs:1929-2070 quantize_sq8_and_assign_global_d0_reference, the
 * assignment half (the caller quantizes rows and leaders with
 * oracle_quantize_sq8, P/dco_sq_int8.rs:1994-2035): for every row the SQ8
 * distance to every leader (sq_int8_approx_l2, P/dco_sq_int8.rs:2950-2965 =
 * oracle_sq8_l2_from_dot), the candidates ordered by stable_distance_order on
 * (distance, leader id) (P/mod.rs:417-428), the first fanout leader INDICES
 * kept, best first (P/dco_sq_int8.rs:2037-2061).
 *
 * The reference orders all candidates with sort_unstable_by under the eps/id
 * rule.  Restated as bounded sequential insertion in ascending leader index
 * under the same rule (insert_topk): where the rule orders the row's
 * candidates consistently the two agree; where eps-tie chains make it
 * inconsistent the sort's result depends on its internal comparison order,
 * and the sequential form is the one defined here (the same rule as the leaf
 * path).  A leader id repeated within eps keeps the earlier index first.
 */
static inline void insert_topk_idx(float d, uint32_t id, uint32_t idx, uint32_t k, float* bd,
                                   uint32_t* bi, uint32_t* bx) {
    if (!better(d, id, bd[k - 1], bi[k - 1])) return;
    uint32_t pos = k - 1;
    while (pos > 0 && better(d, id, bd[pos - 1], bi[pos - 1])) {
        bd[pos] = bd[pos - 1];
        bi[pos] = bi[pos - 1];
        bx[pos] = bx[pos - 1];
        --pos;
    }
    bd[pos] = d;
    bi[pos] = id;
    bx[pos] = idx;
}

int oracle_d0_assign_sq8(const int8_t* codes, const float* scales, const float* norms, uint64_t rows,
                         uint32_t padded_dim, const int8_t* leader_codes, const float* leader_scales,
                         const float* leader_norms, const uint32_t* leader_ids, uint32_t leaders,
                         uint32_t fanout, uint32_t* child_ids, float* dists) {
    if (fanout == 0 || fanout > MAX_K || fanout > leaders) return ORACLE_ERR_ARG;
#pragma omp parallel for schedule(dynamic, 64)
    for (int64_t r = 0; r < (int64_t)rows; ++r) {
        float bd[MAX_K];
        uint32_t bi[MAX_K], bx[MAX_K];
        for (uint32_t s = 0; s < fanout; ++s) { bd[s] = EMPTY_DIST; bi[s] = EMPTY_ID; bx[s] = EMPTY_ID; }
        const int8_t* rc = codes + (uint64_t)r * padded_dim;
        for (uint32_t j = 0; j < leaders; ++j) {
            int32_t dot = oracle_sq8_dot(rc, leader_codes + (uint64_t)j * padded_dim, padded_dim);
            float d = oracle_sq8_l2_from_dot(dot, scales[r], norms[r], leader_scales[j], leader_norms[j]);
            insert_topk_idx(d, leader_ids[j], j, fanout, bd, bi, bx);
        }
        for (uint32_t s = 0; s < fanout; ++s) {
            child_ids[(uint64_t)r * fanout + s] = bx[s];
            if (dists) dists[(uint64_t)r * fanout + s] = bd[s];
        }
    }
    return ORACLE_OK;
}

/* ------------------------------------------------ candidate edges --- */

/*
 * P/hash_prune.rs:2208-2232 fill_sketch_row: out[i*m + h] = sum over axes in
 * order of x[i][a] * planes[h][a], f32, `acc += a * b` (one rounding each).
 */
void oracle_sketch_rows(const float* x, uint64_t rows, uint32_t dim, const float* planes, uint32_t m,
                        float* out) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)rows; ++i) {
        const float* xi = x + (uint64_t)i * dim;
        for (uint32_t h = 0; h < m; ++h) {
            const float* ph = planes + (uint64_t)h * dim;
            float acc = 0.0f;
            for (uint32_t a = 0; a < dim; ++a) {
                float prod = xi[a] * ph[a];
                acc = acc + prod;
            }
            out[(uint64_t)i * m + h] = acc;
        }
    }
}

/* P/hash_prune.rs:2239-2251 compute_hash: bit b = (c[b] - p[b] >= 0). */
uint32_t oracle_compute_hash(const float* sketch_p, const float* sketch_c, uint32_t m_bits) {
    uint32_t h = 0;
    for (uint32_t b = 0; b < m_bits; ++b) {
        float diff = sketch_c[b] - sketch_p[b];
        if (diff >= 0.0f) h |= 1u << b;
    }
    return h;
}

/*
 * P/leaf_build.rs:1749-1808 (flush_compact_topk_batch_into_edges without
 * evidence annotation or lune pruning): for each row i and rank r whose id j
 * is not u32::MAX and whose distance d is finite, the edge
 * (point_ids[i] -> j, compute_hash(s_i, s_j), d) then (j -> point_ids[i],
 * compute_hash(s_j, s_i), d).  Sketch rows are indexed by global point id.
 * Returns the edge count (edges written only if it fits `capacity`).
 */
uint64_t oracle_flush_edges(const uint32_t* point_ids, const uint32_t* topk_ids, const float* topk_dists,
                            uint64_t rows, uint32_t k, const float* sketches, uint32_t width,
                            uint32_t m_bits, uint32_t* out_p, uint32_t* out_c, uint16_t* out_hash,
                            float* out_dist, uint64_t capacity) {
    uint64_t e = 0;
    for (uint64_t i = 0; i < rows; ++i) {
        uint32_t pi = point_ids[i];
        const float* si = sketches + (uint64_t)pi * width;
        for (uint32_t r = 0; r < k; ++r) {
            uint32_t j = topk_ids[i * k + r];
            float d = topk_dists[i * k + r];
            if (j == EMPTY_ID || !isfinite(d)) continue;
            const float* sj = sketches + (uint64_t)j * width;
            if (e + 2 <= capacity) {
                out_p[e] = pi; out_c[e] = j; out_hash[e] = (uint16_t)oracle_compute_hash(si, sj, m_bits);
                out_dist[e] = d;
                out_p[e + 1] = j; out_c[e + 1] = pi;
                out_hash[e + 1] = (uint16_t)oracle_compute_hash(sj, si, m_bits); out_dist[e + 1] = d;
            }
            e += 2;
        }
    }
    return e;
}

/* --------------------------------------------------------- assignment --- */

/* CB:5983-5989 gpu_persistent_hash64 (splitmix64 finaliser). */
uint64_t oracle_hash64(uint64_t v) {
    v ^= v >> 30;
    v *= 0xbf58476d1ce4e5b9ull;
    v ^= v >> 27;
    v *= 0x94d049bb133111ebull;
    return v ^ (v >> 31);
}

/* CB:6510-6520 gpu_persistent_assignment_tie_key. */
uint64_t oracle_assignment_tie_key(uint32_t point, uint32_t leader) {
    return oracle_hash64((((uint64_t)point) << 32) ^ (uint64_t)leader ^ 0x9e3779b97f4a7c15ull);
}

/* CB:6524-6578 gpu_persistent_assignment_insert_candidate (hash-keyed ties). */
static void assign_insert(float d, uint32_t point, uint32_t leader, uint32_t leader_slot,
                          uint32_t slots, float* bd, uint32_t* bslot, uint32_t* bleader) {
    if (slots == 0) return;
    float fdelta = d - bd[slots - 1];
    int is_better = d < bd[slots - 1];
    uint64_t ck = 0;
    int ck_ready = 0;
    if (fabsf(fdelta) <= TIE_EPS) {
        ck = oracle_assignment_tie_key(point, leader);
        ck_ready = 1;
        uint64_t fk = oracle_assignment_tie_key(point, bleader[slots - 1]);
        is_better = ck < fk || (ck == fk && leader < bleader[slots - 1]);
    }
    if (!is_better) return;
    uint32_t pos = slots - 1;
    while (pos > 0) {
        float pdelta = d - bd[pos - 1];
        int before = d < bd[pos - 1];
        if (fabsf(pdelta) <= TIE_EPS) {
            if (!ck_ready) { ck = oracle_assignment_tie_key(point, leader); ck_ready = 1; }
            uint64_t pk = oracle_assignment_tie_key(point, bleader[pos - 1]);
            before = ck < pk || (ck == pk && leader < bleader[pos - 1]);
        }
        if (!before) break;
        bd[pos] = bd[pos - 1];
        bslot[pos] = bslot[pos - 1];
        bleader[pos] = bleader[pos - 1];
        --pos;
    }
    bd[pos] = d;
    bslot[pos] = leader_slot;
    bleader[pos] = leader;
}

/* CB:6077-6087 gpu_persistent_assignment_dot_fp32: sequential rn(rn(a*b) + acc). */
static float dot_fp32_seq(const float* a, const float* b, uint32_t dim) {
    float s = 0.0f;
    for (uint32_t i = 0; i < dim; ++i) s = s + a[i] * b[i];
    return s;
}

/*
 * Assignment distance per executor:
 *   0 (A0 FP32): CB:13621-13624 / CB:6436-6444, rn(rn(n_p + n_l) + rn(-2 * dot)),
 *                dot sequential over axes (tiled order CB:13829-13842 equals it).
 *   2 (SQ8, uncontracted): n_p + n_l - 2*s_p*s_l*dot with one rounding per op.
 *   3 (SQ8, contracted):   fmaf(-(2*s_p*s_l), dot, n_p + n_l) -- the single FFMA
 *                nvcc's default --fmad=true forms from CB:14676-14678.
 * Clamp <= 0 to 0 in every case.
 */
static float assign_dist(uint32_t mode, const float* x, const float* norms, const int8_t* codes,
                         const float* scales, uint32_t dim, uint32_t padded_dim, uint32_t p,
                         uint32_t l) {
    float d;
    if (mode == 0) {
        float dot = dot_fp32_seq(x + (uint64_t)p * dim, x + (uint64_t)l * dim, dim);
        float nn = norms[p] + norms[l];
        float m2 = -2.0f * dot;
        d = nn + m2;
    } else {
        int32_t idot = oracle_sq8_dot(codes + (uint64_t)p * padded_dim,
                                      codes + (uint64_t)l * padded_dim, padded_dim);
        float nn = norms[p] + norms[l];
        float t = (2.0f * scales[p]) * scales[l];
        if (mode == 3) {
            d = fmaf(-t, (float)idot, nn);
        } else {
            float u = t * (float)idot;
            d = nn - u;
        }
    }
    if (d <= 0.0f) d = 0.0f;
    return d;
}

/*
 * gpu_tessa_assignment_replay (CB:15729-15943) semantics: per task member row,
 * the best 4 leader slots (local_fanout 4, CB:15808) over leaders in ascending
 * slot order, then for rank < r_h: id = global_ids[leader], dist recomputed by
 * the same distance (CB:15916-15940).  Output at task_output_offset + row*r_h + rank.
 */
int oracle_assign(uint32_t mode, const float* x, const float* norms, const int8_t* codes,
                  const float* scales, const uint32_t* global_ids, uint64_t resident_rows,
                  uint32_t dim, uint32_t padded_dim, const uint32_t* members,
                  const uint32_t* leaders, const uint32_t* task_member_offsets,
                  const uint32_t* task_member_counts, const uint32_t* task_leader_offsets,
                  const uint32_t* task_leader_counts, const uint32_t* task_rh,
                  const uint64_t* task_output_offsets, uint32_t task_count, uint32_t* out_ids,
                  float* out_dists) {
    if (mode != 0 && mode != 2 && mode != 3) return ORACLE_ERR_ARG;
    for (uint32_t t = 0; t < task_count; ++t) {
        if (task_rh[t] == 0 || task_rh[t] > 4 || task_leader_counts[t] < task_rh[t]) return ORACLE_ERR_ARG;
        for (uint32_t i = 0; i < task_member_counts[t]; ++i)
            if (members[task_member_offsets[t] + i] >= resident_rows) return ORACLE_ERR_RANGE;
        for (uint32_t i = 0; i < task_leader_counts[t]; ++i)
            if (leaders[task_leader_offsets[t] + i] >= resident_rows) return ORACLE_ERR_RANGE;
    }
    for (uint32_t t = 0; t < task_count; ++t) {
        const uint32_t* tm = members + task_member_offsets[t];
        const uint32_t* tl = leaders + task_leader_offsets[t];
        uint32_t nl = task_leader_counts[t], rh = task_rh[t];
#pragma omp parallel for schedule(static)
        for (int64_t row = 0; row < (int64_t)task_member_counts[t]; ++row) {
            uint32_t p = tm[row];
            float bd[4];
            uint32_t bs[4], bl[4];
            for (int s = 0; s < 4; ++s) { bd[s] = EMPTY_DIST; bs[s] = EMPTY_ID; bl[s] = EMPTY_ID; }
            for (uint32_t slot = 0; slot < nl; ++slot) {
                uint32_t l = tl[slot];
                float d = assign_dist(mode, x, norms, codes, scales, dim, padded_dim, p, l);
                assign_insert(d, p, l, slot, 4, bd, bs, bl);
            }
            for (uint32_t rank = 0; rank < rh; ++rank) {
                uint64_t o = task_output_offsets[t] + (uint64_t)row * rh + rank;
                uint32_t slot = bs[rank];
                if (slot >= nl) { out_ids[o] = EMPTY_ID; out_dists[o] = EMPTY_DIST; continue; }
                uint32_t l = tl[slot];
                out_ids[o] = global_ids[l];
                out_dists[o] = assign_dist(mode, x, norms, codes, scales, dim, padded_dim, p, l);
            }
        }
    }
    return ORACLE_OK;
}

int oracle_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void oracle_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}
