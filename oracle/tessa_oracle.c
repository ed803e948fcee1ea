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

/*
 * Both hashes of every (row, rank) slot (the inputs flush_compact_topk_batch_into_edges
 * computes per edge, P/leaf_build.rs:1749-1808): hash_fwd = compute_hash(s_i, s_j),
 * hash_rev = compute_hash(s_j, s_i), i = point_ids[row], j = topk_ids[row*k+rank];
 * 0 for empty slots.
 */
void oracle_slot_hashes(const uint32_t* point_ids, const uint32_t* topk_ids, uint64_t rows, uint32_t k,
                        const float* sketches, uint32_t width, uint32_t m_bits, uint16_t* hash_fwd,
                        uint16_t* hash_rev) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)rows; ++i) {
        const float* si = sketches + (uint64_t)point_ids[i] * width;
        for (uint32_t r = 0; r < k; ++r) {
            uint64_t s = (uint64_t)i * k + r;
            uint32_t j = topk_ids[s];
            if (j == EMPTY_ID) { hash_fwd[s] = 0; hash_rev[s] = 0; continue; }
            const float* sj = sketches + (uint64_t)j * width;
            hash_fwd[s] = (uint16_t)oracle_compute_hash(si, sj, m_bits);
            hash_rev[s] = (uint16_t)oracle_compute_hash(sj, si, m_bits);
        }
    }
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

/* ------------------------------------------ subtree partition (D1+) --- */

/*
 * The recursive leader partition of one or more subtree tasks, as the
 * reference's persistent kernel gpu_persistent_subtree_topk runs it
 * (CB:16336-17381), restated sequentially.  A task is a list of resident rows
 * (ascending); inside it rows are named by their position (the reference's
 * subtree-local resident ids), which the leader sampler and the assignment tie
 * key hash.  Two node paths:
 *   small (process_node, CB:12648-13048): nodes of at most leaf_max rows that
 *     still split because they are a subtree root with fanout_second > 1 and
 *     n * fanout_second <= small_node_limit -- hash bottom-k leaders, up to six
 *     attempts, children below leaf_min merged;
 *   large (stage_large_node + process_large_task_cta, CB:12456-12646 and
 *     CB:15047-15727): every other node above leaf_max -- leaders at evenly
 *     spaced positions, retries with the span sampler (CB:5991-6017), a
 *     balanced even/odd split when no retry is left.
 * Children of at most leaf_max rows are leaves; larger ones are queued one
 * level deeper with seed ^ child * 0x94d049bb133111eb ^ (len << 23).
 *
 * Order.  The reference scatters a large node's rows into its children with
 * atomicAdd (CB:15615-15626), so child row order -- and with it the positional
 * leaders of deeper nodes -- differs from run to run.  The canonical order here
 * is the sequential one: rows in ascending position, fanout slots in rank order
 * (the same order the small path's sort gives).  Rows of every node therefore
 * stay ascending.  The work is organised in rounds (every queued node once per
 * round; a node that retries is queued again with its next attempt), the order
 * in which the GPU driver runs it, so leaves come out in the same order.
 *
 * Arithmetic: SQ8 assignment distance in the contracted form (CB:14676-14678),
 * the hash-tie insertion over local_fanout slots (CB:6524-6578), leader count
 * round(psamp * n) formed as fmaf(psamp, n, 0.5f) (nvcc contracts
 * CB:12761 / CB:12566 the same way).
 */
#define SUBTREE_ERR_OVERSIZED (-10)   /* GPU_PERSISTENT_OVERSIZED_TERMINAL_NODE */
#define SUBTREE_ERR_LEADERS (-11)     /* GPU_PERSISTENT_LEADER_OVERFLOW */
#define SUBTREE_ERR_FANOUT (-12)      /* GPU_PERSISTENT_FANOUT_OVER_32 */
#define SUBTREE_ERR_ROWS (-13)        /* GPU_PERSISTENT_QUEUE_ROW_OVERFLOW */
#define SUBTREE_ERR_CAPACITY (-14)    /* output capacity exceeded */
#define SUBTREE_ERR_NOMEM (-15)

/* CB:7044-7075 gpu_persistent_adaptive_psamp_fraction */
float oracle_adaptive_psamp(float base, uint32_t n, uint32_t depth) {
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

/* CB:7082-7101 gpu_persistent_meaningful_split */
static int meaningful_split(uint32_t parent, uint32_t max_child, uint32_t terminal) {
    if (parent <= terminal || max_child <= terminal) return 1;
    if (max_child >= parent) return 0;
    uint32_t min_shrink = parent >> 5;
    if (min_shrink < 32u) min_shrink = 32u;
    if (min_shrink >= parent) min_shrink = 1u;
    return max_child + min_shrink <= parent;
}

static uint32_t leader_count(float psamp, uint32_t n, uint32_t max_leaders) {
    uint32_t b = (uint32_t)fmaf(psamp, (float)n, 0.5f);
    if (b < 2u) b = 2u;
    if (b > max_leaders) b = max_leaders;
    return b;
}

typedef struct {
    uint32_t task, off, n, depth, attempt, num;
    uint64_t seed;
} st_node;

typedef struct {
    const int8_t* codes;
    const float* scales;
    const float* norms;
    uint32_t pd;
    const uint32_t* members;   /* resident rows of all tasks */
    const uint64_t* task_off;
    /* parameters */
    uint32_t leaf_max, leaf_min, max_depth, max_leaders, fanout_second, root_depth, small_limit;
    float psamp;
    /* outputs */
    uint32_t* leaf_rows;
    uint64_t leaf_rows_cap, leaf_rows_len;
    uint64_t* leaf_starts;
    uint32_t* leaf_sizes;
    uint32_t* leaf_tasks;
    uint64_t leaf_cap, leaf_len;
} st_ctx;

typedef struct {
    uint32_t* rows;
    uint64_t len, cap;
    st_node* nodes;
    uint64_t n, ncap;
} st_round;

static int st_queue(st_round* r, st_node nd, const uint32_t* rows) {
    if (r->n == r->ncap) {
        uint64_t ncap = r->ncap * 2 + 16;
        st_node* a = (st_node*)realloc(r->nodes, ncap * sizeof(st_node));
        if (!a) return SUBTREE_ERR_NOMEM;
        r->nodes = a;
        r->ncap = ncap;
    }
    if (r->len + nd.n > r->cap) {
        uint64_t cap = (r->cap + nd.n) * 2;
        uint32_t* b = (uint32_t*)realloc(r->rows, cap * sizeof(uint32_t));
        if (!b) return SUBTREE_ERR_NOMEM;
        r->rows = b;
        r->cap = cap;
    }
    nd.off = (uint32_t)r->len;
    memcpy(r->rows + r->len, rows, sizeof(uint32_t) * nd.n);
    r->len += nd.n;
    r->nodes[r->n++] = nd;
    return ORACLE_OK;
}

static int st_emit_leaf(st_ctx* c, uint32_t task, const uint32_t* local, uint32_t n) {
    if (c->leaf_len >= c->leaf_cap || c->leaf_rows_len + n > c->leaf_rows_cap) return SUBTREE_ERR_CAPACITY;
    const uint32_t* tm = c->members + c->task_off[task];
    for (uint32_t i = 0; i < n; ++i) c->leaf_rows[c->leaf_rows_len + i] = tm[local[i]];
    c->leaf_starts[c->leaf_len] = c->leaf_rows_len;
    c->leaf_sizes[c->leaf_len] = n;
    c->leaf_tasks[c->leaf_len] = task;
    c->leaf_len++;
    c->leaf_rows_len += n;
    return ORACLE_OK;
}

/* Best local_fanout leader slots of one row (tie ids are local ids). */
static void st_assign_row(const st_ctx* c, uint32_t task, uint32_t point, const uint32_t* leaders,
                          uint32_t num, uint32_t lf, uint32_t* out_slots) {
    const uint32_t* tm = c->members + c->task_off[task];
    float bd[4];
    uint32_t bs[4], bl[4];
    for (int s = 0; s < 4; ++s) { bd[s] = EMPTY_DIST; bs[s] = EMPTY_ID; bl[s] = EMPTY_ID; }
    uint32_t rp = tm[point];
    for (uint32_t slot = 0; slot < num; ++slot) {
        uint32_t rl = tm[leaders[slot]];
        float d = assign_dist(3, NULL, c->norms, c->codes, c->scales, 0, c->pd, rp, rl);
        assign_insert(d, point, leaders[slot], slot, lf, bd, bs, bl);
    }
    for (uint32_t k = 0; k < lf; ++k) out_slots[k] = bs[k];
}

/* merge two ascending lists into out (ascending, duplicates dropped) */
static uint32_t merge_unique(const uint32_t* a, uint32_t na, const uint32_t* b, uint32_t nb, uint32_t* out) {
    uint32_t i = 0, j = 0, o = 0;
    while (i < na || j < nb) {
        uint32_t v;
        if (j >= nb || (i < na && a[i] <= b[j])) v = a[i++];
        else v = b[j++];
        if (o == 0 || out[o - 1] != v) out[o++] = v;
    }
    return o;
}

static uint64_t child_seed(uint64_t seed, uint32_t child, uint32_t len) {
    return seed ^ ((uint64_t)child * 0x94d049bb133111ebull) ^ (((uint64_t)len) << 23);
}

/* process_node (CB:12648-13048) for a node that splits on the small path. */
static int st_small(st_ctx* c, const st_node* nd, const uint32_t* rows, st_round* next) {
    uint32_t n = nd->n;
    uint32_t depth = nd->depth;
    uint32_t rd = depth >= c->root_depth ? depth - c->root_depth : 0u;
    uint32_t terminal = c->leaf_max;
    if (depth >= c->max_depth) return SUBTREE_ERR_OVERSIZED;
    uint32_t max_leaders = c->max_leaders < n ? c->max_leaders : n;
    if (max_leaders < 2u) max_leaders = 2u;
    if (max_leaders > 128u) return SUBTREE_ERR_LEADERS;
    uint32_t base = leader_count(oracle_adaptive_psamp(c->psamp, n, depth), n, max_leaders);
    uint32_t requested = rd == 0u ? c->fanout_second : 1u;
    if (requested < 1u) requested = 1u;
    if (requested > 4u) return SUBTREE_ERR_FANOUT;
    uint32_t leaders[128], counts[128], starts[128], writes[128];
    uint32_t child_off[129], child_cnt[129];
    uint32_t* slots = (uint32_t*)malloc(sizeof(uint32_t) * 4u * n);
    uint32_t* clustered = (uint32_t*)malloc(sizeof(uint32_t) * 4096u);
    uint32_t* merged = (uint32_t*)malloc(sizeof(uint32_t) * 4096u);
    uint32_t* small = (uint32_t*)malloc(sizeof(uint32_t) * 4096u);
    uint32_t* tmp = (uint32_t*)malloc(sizeof(uint32_t) * 8192u);
    int rc = ORACLE_OK, ok = 0;
    uint32_t nchild = 0;
    if (!slots || !clustered || !merged || !small || !tmp) { rc = SUBTREE_ERR_NOMEM; goto done; }
    for (uint32_t attempt = 0; attempt < 6u; ++attempt) {
        uint32_t num = base << attempt;
        if (num > max_leaders || (base << attempt) >> attempt != base) num = max_leaders;
        uint64_t scores[128];
        for (uint32_t s = 0; s < num; ++s) { leaders[s] = 0xffffffffu; scores[s] = ~0ull; }
        for (uint32_t i = 0; i < n; ++i) {
            uint32_t point = rows[i];
            uint64_t key = oracle_hash64(nd->seed ^ ((uint64_t)attempt * 0xbf58476d1ce4e5b9ull) ^
                                         (((uint64_t)depth) << 19) ^ (((uint64_t)i) << 7) ^
                                         (((uint64_t)point) << 31));
            uint32_t ins = num;
            for (uint32_t p = 0; p < num; ++p)
                if (key < scores[p] || (key == scores[p] && point < leaders[p])) { ins = p; break; }
            if (ins < num) {
                for (uint32_t p = num - 1; p > ins; --p) { scores[p] = scores[p - 1]; leaders[p] = leaders[p - 1]; }
                scores[ins] = key;
                leaders[ins] = point;
            }
        }
        uint32_t lf = requested < num ? requested : num;
        for (uint32_t s = 0; s < num; ++s) counts[s] = 0;
        for (uint32_t i = 0; i < n; ++i) {
            st_assign_row(c, nd->task, rows[i], leaders, num, lf, slots + (uint64_t)i * lf);
            for (uint32_t k = 0; k < lf; ++k) {
                uint32_t s = slots[(uint64_t)i * lf + k];
                if (s >= num) { rc = SUBTREE_ERR_ROWS; goto done; }
                counts[s]++;
            }
        }
        uint32_t running = 0;
        for (uint32_t s = 0; s < num; ++s) { starts[s] = running; writes[s] = running; running += counts[s]; }
        if (running > 4096u) { rc = SUBTREE_ERR_ROWS; goto done; }
        for (uint32_t i = 0; i < n; ++i)
            for (uint32_t k = 0; k < lf; ++k) clustered[writes[slots[(uint64_t)i * lf + k]]++] = rows[i];
        nchild = 0;
        uint32_t merged_rows = 0, small_len = 0, max_child = 0;
        for (uint32_t s = 0; s < num; ++s) {
            uint32_t cnt = counts[s];
            if (cnt == 0) continue;
            const uint32_t* seg = clustered + starts[s];  /* ascending, distinct */
            if (cnt < c->leaf_min) {
                uint32_t m = merge_unique(small, small_len, seg, cnt, tmp);
                memcpy(small, tmp, sizeof(uint32_t) * m);
                small_len = m;
                if (small_len >= c->leaf_min) {
                    memcpy(merged + merged_rows, small, sizeof(uint32_t) * small_len);
                    child_off[nchild] = merged_rows;
                    child_cnt[nchild] = small_len;
                    merged_rows += small_len;
                    if (small_len > max_child) max_child = small_len;
                    nchild++;
                    small_len = 0;
                }
            } else {
                child_off[nchild] = merged_rows;
                child_cnt[nchild] = cnt;
                memcpy(merged + merged_rows, seg, sizeof(uint32_t) * cnt);
                merged_rows += cnt;
                if (cnt > max_child) max_child = cnt;
                nchild++;
            }
        }
        if (small_len > 0 && nchild > 0) {
            uint32_t last = nchild - 1;
            if (child_cnt[last] + small_len <= terminal) {
                uint32_t m = merge_unique(merged + child_off[last], child_cnt[last], small, small_len, tmp);
                memcpy(merged + child_off[last], tmp, sizeof(uint32_t) * m);
                merged_rows = child_off[last] + m;
                child_cnt[last] = m;
                if (m > max_child) max_child = m;
                small_len = 0;
            }
        }
        if (small_len > 0) {
            memcpy(merged + merged_rows, small, sizeof(uint32_t) * small_len);
            child_off[nchild] = merged_rows;
            child_cnt[nchild] = small_len;
            merged_rows += small_len;
            if (small_len > max_child) max_child = small_len;
            nchild++;
        }
        if (nchild > 1 && meaningful_split(n, max_child, terminal)) { ok = 1; break; }
        if (num >= max_leaders) break;
    }
    if (!ok) {
        if (n > terminal) { rc = SUBTREE_ERR_OVERSIZED; goto done; }
        rc = st_emit_leaf(c, nd->task, rows, n);
        goto done;
    }
    for (uint32_t ci = 0; ci < nchild && rc == ORACLE_OK; ++ci) {
        uint32_t len = child_cnt[ci];
        const uint32_t* cr = merged + child_off[ci];
        if (len == 0) continue;
        if (len <= terminal) {
            rc = st_emit_leaf(c, nd->task, cr, len);
        } else if (depth + 1u >= c->max_depth) {
            rc = SUBTREE_ERR_OVERSIZED;
        } else {
            st_node ch = {nd->task, 0u, len, depth + 1u, 0u, 0u, child_seed(nd->seed, ci, len)};
            rc = st_queue(next, ch, cr);
        }
    }
done:
    free(slots); free(clustered); free(merged); free(small); free(tmp);
    return rc;
}

/* gpu_persistent_sample_large_retry_leaders (CB:5991-6017) */
static void st_retry_leaders(const uint32_t* rows, uint32_t n, uint32_t num, uint64_t seed, uint32_t attempt,
                             uint32_t* leaders) {
    for (uint32_t s = 0; s < num; ++s) {
        uint32_t b = (uint32_t)(((uint64_t)s * n) / num);
        uint32_t e = (uint32_t)(((uint64_t)(s + 1u) * n) / num);
        if (e <= b) e = b + 1u;
        uint32_t span = e - b;
        uint64_t key = oracle_hash64(seed ^ ((uint64_t)attempt * 0xd6e8feb86659fd93ull) ^
                                     ((uint64_t)s * 0x9e3779b97f4a7c15ull));
        leaders[s] = rows[b + (uint32_t)(key % span)];
    }
}

/*
 * Partition the tasks into leaves.  params = {leaf_max, leaf_min, max_depth,
 * max_leaders, fanout_second, root_depth, small_node_limit}; task t has rows
 * members[task_offsets[t] .. + task_counts[t]) (ascending resident ids) and
 * seed task_seeds[t].  Leaves are written as resident ids in round order;
 * returns the leaf count or a negative error.  out_stats (may be NULL) gets
 * {rounds, large-node assignments, retries, balanced splits, small nodes}.
 */
int64_t oracle_subtree_partition(const int8_t* codes, const float* scales, const float* norms,
                                 uint32_t padded_dim, const uint32_t* members, const uint64_t* task_offsets,
                                 const uint32_t* task_counts, const uint64_t* task_seeds, uint32_t task_count,
                                 const uint32_t* params, float psamp, uint32_t* leaf_rows, uint64_t leaf_rows_cap,
                                 uint64_t* leaf_starts, uint32_t* leaf_sizes, uint32_t* leaf_tasks,
                                 uint64_t leaf_cap, uint64_t* out_stats) {
    st_ctx c;
    memset(&c, 0, sizeof c);
    c.codes = codes; c.scales = scales; c.norms = norms; c.pd = padded_dim;
    c.members = members; c.task_off = task_offsets;
    c.leaf_max = params[0]; c.leaf_min = params[1]; c.max_depth = params[2];
    c.max_leaders = params[3] < 128u ? params[3] : 128u;
    c.fanout_second = params[4]; c.root_depth = params[5]; c.small_limit = params[6];
    c.psamp = psamp;
    c.leaf_rows = leaf_rows; c.leaf_rows_cap = leaf_rows_cap;
    c.leaf_starts = leaf_starts; c.leaf_sizes = leaf_sizes; c.leaf_tasks = leaf_tasks; c.leaf_cap = leaf_cap;
    if (c.leaf_max == 0 || c.leaf_min == 0 || c.leaf_max > c.small_limit) return ORACLE_ERR_ARG;
    uint64_t stats[5] = {0, 0, 0, 0, 0};
    uint64_t cur_len = 0, cur_cap = 16, nn = 0;
    for (uint32_t t = 0; t < task_count; ++t) cur_cap += task_counts[t];
    uint32_t* cur = (uint32_t*)malloc(cur_cap * sizeof(uint32_t));
    st_node* nodes = (st_node*)malloc((task_count + 16) * sizeof(st_node));
    int rc = ORACLE_OK;
    if (!cur || !nodes) { free(cur); free(nodes); return SUBTREE_ERR_NOMEM; }
    for (uint32_t t = 0; t < task_count; ++t) {
        if (task_counts[t] == 0) continue;
        st_node r = {t, (uint32_t)cur_len, task_counts[t], c.root_depth, 0u, 0u, task_seeds[t]};
        for (uint32_t i = 0; i < task_counts[t]; ++i) cur[cur_len + i] = i;
        cur_len += task_counts[t];
        nodes[nn++] = r;
    }
    uint32_t* slots = NULL;
    uint64_t slots_cap = 0;
    while (nn > 0 && rc == ORACLE_OK) {
        stats[0]++;
        st_round next = {NULL, 0, 0, NULL, 0, 0};
        for (uint64_t q = 0; q < nn && rc == ORACLE_OK; ++q) {
            st_node nd = nodes[q];
            const uint32_t* rows = cur + nd.off;
            uint32_t n = nd.n;
            uint32_t rd = nd.depth >= c.root_depth ? nd.depth - c.root_depth : 0u;
            int probe = rd == 0u && c.fanout_second > 1u && n > 1u;
            int probe_over = probe && (uint64_t)n * c.fanout_second > c.small_limit;
            if (n <= c.leaf_max && !probe_over) {
                if (!probe) { rc = st_emit_leaf(&c, nd.task, rows, n); continue; }
                stats[4]++;
                rc = st_small(&c, &nd, rows, &next);
                continue;
            }
            /* large path: stage_large_node (CB:12456-12646) */
            if (nd.depth >= c.max_depth) { rc = SUBTREE_ERR_OVERSIZED; break; }
            uint32_t retry_max = n < 2u ? 2u : n;
            if (retry_max > 128u) retry_max = 128u;
            uint32_t max_leaders = c.max_leaders < retry_max ? c.max_leaders : retry_max;
            if (max_leaders < 2u) max_leaders = 2u;
            uint32_t requested = rd == 0u ? c.fanout_second : 1u;
            if (requested < 1u) requested = 1u;
            if (requested > 4u) { rc = SUBTREE_ERR_FANOUT; break; }
            uint32_t base = leader_count(oracle_adaptive_psamp(c.psamp, n, nd.depth), n, max_leaders);
            uint32_t lf = requested < base ? requested : base;  /* fixed at staging */
            uint32_t num = nd.attempt == 0u ? base : nd.num;
            uint32_t leaders[128], counts[128];
            if (nd.attempt == 0u) {
                for (uint32_t s = 0; s < num; ++s) {
                    uint64_t ord = ((uint64_t)s * n) / num;
                    if (ord >= n) ord = n - 1u;
                    leaders[s] = rows[ord];
                }
            } else {
                st_retry_leaders(rows, n, num, nd.seed, nd.attempt, leaders);
            }
            if (slots_cap < (uint64_t)n * 4u) {
                free(slots);
                slots_cap = (uint64_t)n * 4u;
                slots = (uint32_t*)malloc(slots_cap * sizeof(uint32_t));
                if (!slots) { rc = SUBTREE_ERR_NOMEM; break; }
            }
            stats[1]++;
            for (uint32_t s = 0; s < num; ++s) counts[s] = 0;
#pragma omp parallel for schedule(static)
            for (int64_t i = 0; i < (int64_t)n; ++i)
                st_assign_row(&c, nd.task, rows[i], leaders, num, lf, slots + (uint64_t)i * lf);
            for (uint32_t i = 0; i < n; ++i)
                for (uint32_t k = 0; k < lf; ++k) {
                    uint32_t s = slots[(uint64_t)i * lf + k];
                    if (s < num) counts[s]++;
                }
            uint32_t nonempty = 0, max_child = 0;
            for (uint32_t s = 0; s < num; ++s)
                if (counts[s]) { nonempty++; if (counts[s] > max_child) max_child = counts[s]; }
            int split = nonempty > 1u && meaningful_split(n, max_child, c.leaf_max);
            int balanced = 0;
            if (!split) {
                if (nd.attempt == 0u || num < retry_max) {
                    uint32_t next_num = num;
                    if (nd.attempt > 0u) {
                        uint32_t dbl = num << 1;
                        next_num = (dbl > num && dbl < retry_max) ? dbl : retry_max;
                    }
                    if (next_num > retry_max) next_num = retry_max;
                    /* queued again, same rows, next attempt */
                    st_node again = nd;
                    again.attempt = nd.attempt + 1u;
                    again.num = next_num;
                    rc = st_queue(&next, again, rows);
                    stats[2]++;
                    continue;
                }
                balanced = 1;
                stats[3]++;
            }
            /* children: slot order (balanced: position parity), rows ascending */
            uint32_t nchild = balanced ? 2u : num;
            for (uint32_t ci = 0; ci < nchild && rc == ORACLE_OK; ++ci) {
                uint32_t len = 0;
                uint32_t* buf = (uint32_t*)malloc(sizeof(uint32_t) * (n + 1u));
                if (!buf) { rc = SUBTREE_ERR_NOMEM; break; }
                for (uint32_t i = 0; i < n; ++i) {
                    if (balanced) {
                        if ((i & 1u) == ci) buf[len++] = rows[i];
                    } else {
                        for (uint32_t k = 0; k < lf; ++k)
                            if (slots[(uint64_t)i * lf + k] == ci) { buf[len++] = rows[i]; break; }
                    }
                }
                if (len == 0) { free(buf); continue; }
                if (len <= c.leaf_max) {
                    rc = st_emit_leaf(&c, nd.task, buf, len);
                } else if (nd.depth + 1u >= c.max_depth) {
                    rc = SUBTREE_ERR_OVERSIZED;
                } else {
                    st_node ch = {nd.task, 0u, len, nd.depth + 1u, 0u, 0u, child_seed(nd.seed, ci, len)};
                    rc = st_queue(&next, ch, buf);
                }
                free(buf);
            }
        }
        free(cur);
        free(nodes);
        cur = next.rows;
        cur_len = next.len;
        nodes = next.nodes;
        nn = next.n;
    }
    free(cur);
    free(nodes);
    free(slots);
    if (out_stats) memcpy(out_stats, stats, sizeof stats);
    return rc == ORACLE_OK ? (int64_t)c.leaf_len : (int64_t)rc;
}
