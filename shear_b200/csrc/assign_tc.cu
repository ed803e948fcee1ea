// TESSA leader assignment replay, SQ8 source, on the tensor cores (sm_100a).
//
// Same result as assign_kernel<true, LG> (assign.cu): for every member row of
// a frozen task, the int8 dots with the task's leaders, the SQ8 distance
// n_p + n_l - 2*s_p*s_l*dot in the contracted single-FFMA form
// (CB:14676-14678), and the reference's four-slot hash-tie insertion
// (CB:6524-6578) over the leaders in ascending slot order, then the first r_h
// slots as (global id, distance).  Only the dots move to the tensor cores:
// they are exact int32 sums either way, so the results are bit-identical.
//
// The work is a stream of items (128 member rows of one task); the member and
// leader rows are gathered by id, so the kernel is a pipelined gather feeding
// tcgen05.mma.  Warp-specialised, persistent, two CTAs per SM:
//   warps 0-3  producers: walk the items, load each item's metadata chain
//              (work entry -> task -> member and leader ids -> norms, scales,
//              global ids) into a metadata slot, and copy the rows one
//              128-byte K slab at a time into a ring of shared-memory stages,
//              already in the 128-byte swizzled K-major layout the MMA reads
//              (piece j of row r at j ^ (r & 7)).  Thread t copies piece t & 7
//              of rows (t >> 3) + 16u, from row pointers computed once per
//              item; cp.async.mbarrier.arrive hands the completion of a
//              thread's copies to the stage's barrier, so a producer never
//              waits for its own copies and every stage of the ring can be in
//              flight, across item boundaries;
//   warp 8     TMEM owner and MMA issuer: tcgen05.mma.kind::i8, M = 128 rows,
//              N = NB leader slots (the launch's leader count rounded up to 16),
//              K = 32, into one of two accumulator buffers; tcgen05.commit
//              frees each stage and, after an item's last slab, hands the
//              buffer to the epilogue;
//   warps 4-7  epilogue: warp 4 + q reads TMEM lanes 32q..32q+31 (its rows'
//              dots) and runs the distance and the insertion per row, while
//              the MMA fills the other buffer.
// Every wait is bounded; a timed-out or aborted wait raises the CTA's abort
// flag and the error word, and all roles then leave their loops.
#include "common.cuh"
#include "kernels.h"

namespace tessa {
namespace assign {
namespace tc {

constexpr uint32_t kRowsTc = 128;  // member rows per work item (MMA M = TMEM lanes)
constexpr uint32_t kSlabTc = 128;  // K bytes per slab (one 128-byte swizzle atom)
constexpr uint32_t kMmaKTc = 32;
constexpr uint32_t kASlabTc = kRowsTc * kSlabTc;  // 16 KiB
constexpr uint32_t kMaxNB = 128;  // leader slots per MMA (task leader counts above use the SIMT kernel)
constexpr uint32_t kProdThreads = 128;  // warps 0-3
constexpr uint32_t kAccBufs = 4;        // accumulator buffers = metadata slots = epilogue groups
constexpr uint32_t kEpiWarp0 = 4;       // warps 4-19: epilogue group g = warps 4 + 4g .. 7 + 4g
constexpr uint32_t kMmaWarp = 4 + 4 * kAccBufs;
constexpr uint32_t kThreadsTc = (kMmaWarp + 1) * 32;
constexpr uint32_t kSmemPerCta = 232448u;  // one CTA per SM

template <uint32_t NB>
struct Geom {
  static constexpr uint32_t kStage = kASlabTc + NB * kSlabTc;  // A slab then B slab, multiples of 1 KiB
  // metadata slot: per row point/norm/scale, per leader slot id/gid/norm/scale, item fields
  static constexpr uint32_t kMeta = kRowsTc * 12u + NB * 16u + 32u;
  static constexpr uint32_t kMetaSlots = kAccBufs;
  static constexpr uint32_t kBars = 256u;
  static constexpr uint32_t kFixed = 1024u + kMetaSlots * kMeta + kBars;
  static constexpr uint32_t kStages = (kSmemPerCta - kFixed) / kStage < 8u ? (kSmemPerCta - kFixed) / kStage : 8u;
  static constexpr uint32_t kSmem = 1024u + kStages * kStage + kMetaSlots * kMeta + kBars;
  static constexpr uint32_t kTmemCols = kAccBufs * NB <= 64u ? 64u : (kAccBufs * NB <= 128u ? 128u : (kAccBufs * NB <= 256u ? 256u : 512u));
  static_assert(kStages >= 3, "ring too shallow");
  static_assert(kSmem <= kSmemPerCta, "shared memory");
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

struct Top4 {
  float d[4];
  uint32_t s[4], l[4];
};

// CB:6524-6578 with slots = 4 (as assign.cu's insert4).  Out of line: it is
// only reached for a candidate within the 2e-5 tie window of a held slot.
__device__ __noinline__ Top4 insert4_ties(Top4 t, float d, uint32_t point, uint32_t leader, uint32_t slot) {
  float (&bd)[4] = t.d;
  uint32_t (&bs)[4] = t.s;
  uint32_t (&bl)[4] = t.l;
  bool better = d < bd[3];
  uint64_t ck = 0;
  bool ck_ready = false;
  if (fabsf(__fsub_rn(d, bd[3])) <= 2.0e-5f) {
    ck = tie_key(point, leader);
    ck_ready = true;
    const uint64_t fk = tie_key(point, bl[3]);
    better = ck < fk || (ck == fk && leader < bl[3]);
  }
  if (!better) return t;
  int pos = 3;
#pragma unroll
  for (int j = 3; j >= 1; --j) {
    if (pos != j) break;
    bool before = d < bd[j - 1];
    if (fabsf(__fsub_rn(d, bd[j - 1])) <= 2.0e-5f) {
      if (!ck_ready) {
        ck = tie_key(point, leader);
        ck_ready = true;
      }
      const uint64_t pk = tie_key(point, bl[j - 1]);
      before = ck < pk || (ck == pk && leader < bl[j - 1]);
    }
    if (!before) break;
    bd[j] = bd[j - 1];
    bs[j] = bs[j - 1];
    bl[j] = bl[j - 1];
    pos = j - 1;
  }
#pragma unroll
  for (int j = 0; j < 4; ++j)
    if (j == pos) {
      bd[j] = d;
      bs[j] = slot;
      bl[j] = leader;
    }
  return t;
}

// The same insertion.  A candidate more than 2e-5 from every held slot
// compares by distance alone against each of them (no tie key is consulted),
// so it is placed by a short branch-free network; otherwise the full rule runs.
__device__ __forceinline__ void insert4(float d, uint32_t point, uint32_t leader, uint32_t slot, float (&bd)[4],
                                        uint32_t (&bs)[4], uint32_t (&bl)[4]) {
  const bool near = fabsf(__fsub_rn(d, bd[0])) <= 2.0e-5f || fabsf(__fsub_rn(d, bd[1])) <= 2.0e-5f ||
                    fabsf(__fsub_rn(d, bd[2])) <= 2.0e-5f || fabsf(__fsub_rn(d, bd[3])) <= 2.0e-5f;
  if (near) {
    Top4 t;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      t.d[k] = bd[k];
      t.s[k] = bs[k];
      t.l[k] = bl[k];
    }
    t = insert4_ties(t, d, point, leader, slot);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      bd[k] = t.d[k];
      bs[k] = t.s[k];
      bl[k] = t.l[k];
    }
    return;
  }
  if (!(d < bd[3])) return;
  const bool c0 = d < bd[0], c1 = d < bd[1], c2 = d < bd[2];
  bd[3] = c2 ? bd[2] : d;
  bs[3] = c2 ? bs[2] : slot;
  bl[3] = c2 ? bl[2] : leader;
  bd[2] = c1 ? bd[1] : (c2 ? d : bd[2]);
  bs[2] = c1 ? bs[1] : (c2 ? slot : bs[2]);
  bl[2] = c1 ? bl[1] : (c2 ? leader : bl[2]);
  bd[1] = c0 ? bd[0] : (c1 ? d : bd[1]);
  bs[1] = c0 ? bs[0] : (c1 ? slot : bs[1]);
  bl[1] = c0 ? bl[0] : (c1 ? leader : bl[1]);
  bd[0] = c0 ? d : bd[0];
  bs[0] = c0 ? slot : bs[0];
  bl[0] = c0 ? leader : bl[0];
}

// CB:6524-6578 with a list of n <= 4 slots (the subtree partition keeps
// local_fanout slots, CB:6618-6698): the candidate is tested against slot
// n - 1 first, then moved up while it beats the slot above.
__device__ __forceinline__ void insertn(float d, uint32_t point, uint32_t leader, uint32_t slot, uint32_t n,
                                        float (&bd)[4], uint32_t (&bs)[4], uint32_t (&bl)[4]) {
  const uint32_t last = n - 1u;
  float dl = bd[0];
  uint32_t ll = bl[0];
#pragma unroll
  for (uint32_t j = 1; j < 4; ++j)
    if (j == last) {
      dl = bd[j];
      ll = bl[j];
    }
  bool better = d < dl;
  uint64_t ck = 0;
  bool ck_ready = false;
  if (fabsf(__fsub_rn(d, dl)) <= 2.0e-5f) {
    ck = tie_key(point, leader);
    ck_ready = true;
    const uint64_t fk = tie_key(point, ll);
    better = ck < fk || (ck == fk && leader < ll);
  }
  if (!better) return;
  uint32_t pos = last;
#pragma unroll
  for (uint32_t j = 3; j >= 1; --j) {
    if (j > last || pos != j) continue;
    bool before = d < bd[j - 1];
    if (fabsf(__fsub_rn(d, bd[j - 1])) <= 2.0e-5f) {
      if (!ck_ready) {
        ck = tie_key(point, leader);
        ck_ready = true;
      }
      const uint64_t pk = tie_key(point, bl[j - 1]);
      before = ck < pk || (ck == pk && leader < bl[j - 1]);
    }
    if (!before) continue;
    bd[j] = bd[j - 1];
    bs[j] = bs[j - 1];
    bl[j] = bl[j - 1];
    pos = j - 1;
  }
#pragma unroll
  for (uint32_t j = 0; j < 4; ++j)
    if (j == pos) {
      bd[j] = d;
      bs[j] = slot;
      bl[j] = leader;
    }
}

// d[j] for a run-time j < 16 (a four-level select tree).
__device__ __forceinline__ float select16(const float (&d)[16], uint32_t j) {
  float a8[8], b4[4];
#pragma unroll
  for (uint32_t i = 0; i < 8; ++i) a8[i] = (j & 1u) ? d[2 * i + 1] : d[2 * i];
#pragma unroll
  for (uint32_t i = 0; i < 4; ++i) b4[i] = (j & 2u) ? a8[2 * i + 1] : a8[2 * i];
  const float c0 = (j & 4u) ? b4[1] : b4[0], c1 = (j & 4u) ? b4[3] : b4[2];
  return (j & 8u) ? c1 : c0;
}

__device__ __forceinline__ void cp_async16(uint32_t smem_addr, const void* gmem, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr), "l"(gmem), "r"(src_bytes)
               : "memory");
}
// Arrive on `bar` once every cp.async this thread issued before has landed
// (the arrival is part of the barrier's expected count).
__device__ __forceinline__ void cp_async_mbar_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// 32 lanes x 16 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

template <uint32_t NB>
struct MetaSlot {
  uint32_t pt[kRowsTc];  // member row of each tile row (0xffffffff: none)
  float np[kRowsTc];
  float sp[kRowsTc];
  uint32_t lid[NB];      // leader row of each slot (0xffffffff: none)
  uint32_t lg[NB];
  // per leader pair (2i, 2i + 1): norm, norm, scale, scale (one 16-byte load
  // for two leaders); a missing leader has norm +inf, so its distance is +inf
  float lnls[2 * NB];
  uint32_t task, rh, nl, r0;
  uint64_t tout;
  uint32_t pad[2];
};

// One item's producer-side metadata: the task, this thread's metadata row and
// leader slot, and the member and leader rows it copies.  Loaded as a chain of
// dependent loads (steps 0..3), so the next item's chain is walked one step
// per slab while the current item's slabs are issued.
template <uint32_t NB>
struct ProdMeta {
  uint32_t task, r0, moff, mcnt, loff, nl, rh;
  uint64_t tout;
  uint32_t pt, lid, lg;
  float np, sp, ln, ls;
  uint32_t crow[8];       // member rows (t >> 3) + 16u of the item (0xffffffff: none)
  uint32_t lrow[NB / 16];  // leader rows (t >> 3) + 16v of the task
};

template <uint32_t NB>
__device__ __forceinline__ void prod_step(const Params& p, uint32_t item, uint32_t step, ProdMeta<NB>& m,
                                          uint32_t t) {
  constexpr uint32_t kNone = 0xffffffffu;
  const uint32_t row0 = t >> 3;
  if (step == 0) {
    const uint2 w = p.work[item];
    m.task = w.x;
    m.r0 = w.y;
  } else if (step == 1) {
    m.moff = p.t_moff[m.task];
    m.mcnt = p.t_mcnt[m.task];
    m.loff = p.t_loff[m.task];
    m.nl = p.t_lcnt[m.task];
    m.rh = p.t_rh[m.task];
    m.tout = p.t_out[m.task];
  } else if (step == 2) {
    const uint32_t r = m.r0 + t;
    m.pt = r < m.mcnt ? p.members[m.moff + r] : kNone;
    m.lid = (t < NB && t < m.nl) ? p.leaders[m.loff + t] : kNone;
#pragma unroll
    for (uint32_t u = 0; u < 8; ++u) {
      const uint32_t rr = m.r0 + row0 + 16u * u;
      m.crow[u] = rr < m.mcnt ? p.members[m.moff + rr] : kNone;
    }
#pragma unroll
    for (uint32_t v = 0; v < NB / 16; ++v) {
      const uint32_t lr = row0 + 16u * v;
      m.lrow[v] = lr < m.nl ? p.leaders[m.loff + lr] : kNone;
    }
  } else {
    // Ids at or past resident_rows are reported (each row and leader slot by
    // the thread that owns its metadata) and dropped.
    if (m.pt != kNone && m.pt >= p.resident_rows) {
      atomicOr(p.err_word, TESSA_DEVERR_BAD_ROW);
      m.pt = kNone;
    }
    if (m.lid != kNone && m.lid >= p.resident_rows) {
      atomicOr(p.err_word, TESSA_DEVERR_BAD_ROW);
      m.lid = kNone;
    }
#pragma unroll
    for (uint32_t u = 0; u < 8; ++u)
      if (m.crow[u] >= p.resident_rows) m.crow[u] = kNone;
#pragma unroll
    for (uint32_t v = 0; v < NB / 16; ++v)
      if (m.lrow[v] >= p.resident_rows) m.lrow[v] = kNone;
    m.np = m.pt != kNone ? p.sq8_norms[m.pt] : 0.f;
    m.sp = m.pt != kNone ? p.scales[m.pt] : 0.f;
    m.ln = m.lid != kNone ? p.sq8_norms[m.lid] : INFINITY;
    m.ls = m.lid != kNone ? p.scales[m.lid] : 0.f;
    m.lg = (m.lid != kNone && !p.out_slots) ? p.global_ids[m.lid] : 0u;
    // slot mode: the insertion hashes subtree-local ids
    if (p.member_tie && m.pt != kNone) m.pt = p.member_tie[m.moff + m.r0 + t];
    if (p.leader_tie && m.lid != kNone) m.lid = p.leader_tie[m.loff + t];
  }
}

template <uint32_t NB, bool SLOTS>
__global__ void __launch_bounds__(kThreadsTc, 1) assign_tc_kernel(const Params p) {
  using G = Geom<NB>;
  static_assert(sizeof(MetaSlot<NB>) == G::kMeta, "metadata slot size");
  constexpr uint32_t S = G::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023u) & ~uintptr_t(1023u));
  uint8_t* ring = base;
  MetaSlot<NB>* meta = reinterpret_cast<MetaSlot<NB>*>(ring + S * G::kStage);
  uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(meta) + G::kMetaSlots * G::kMeta);
  uint64_t* full = bars;                 // [S] stage copies landed (128 producer arrivals)
  uint64_t* empty = bars + 8;            // [S] stage read by its MMAs
  uint64_t* acc_full = bars + 16;        // [kAccBufs] buffer's item complete
  uint64_t* acc_empty = bars + 20;       // [kAccBufs] buffer and metadata slot released by the epilogue
  uint64_t* meta_full = bars + 24;       // [kAccBufs] metadata slot written
  uint64_t* done_bar = bars + 28;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 29);
  uint32_t* abort_word = tmem_slot + 1;
  volatile uint32_t* abort_flag = abort_word;

  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31u;
  if (tid == 0) {
    for (uint32_t i = 0; i < S; ++i) {
      mbar_init(&full[i], kProdThreads);
      mbar_init(&empty[i], 1);
    }
    for (uint32_t i = 0; i < kAccBufs; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);
      mbar_init(&meta_full[i], kProdThreads);
    }
    mbar_init(done_bar, 1);
    *abort_word = 0u;
    fence_barrier_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(tmem_slot, G::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t pd = p.padded_dim;
  const uint32_t nslab = (pd + kSlabTc - 1) / kSlabTc;
  const uint32_t ring0 = smem_u32(ring);

  if (warp < kEpiWarp0) {
    // ------------------------------------------------------------ producers
    const uint32_t t = tid;
    const uint32_t piece = t & 7u, row0 = t >> 3;
    const uint32_t swz = (piece ^ (row0 & 7u)) << 4;  // row & 7 == row0 & 7 for rows row0 + 16u
    uint32_t gs = 0;  // slabs issued by this thread
    bool ok = true;
    ProdMeta<NB> cur, nxt;
    if (blockIdx.x < p.num_work)
      for (uint32_t step = 0; step < 4; ++step) prod_step<NB>(p, blockIdx.x, step, cur, t);
    for (uint32_t item = blockIdx.x, li = 0; ok && item < p.num_work; item += gridDim.x, ++li) {
      const uint32_t a = li % kAccBufs;
      const uint32_t next = item + gridDim.x;
      const bool has_next = next < p.num_work;
      // the metadata slot is free once the epilogue released item li - kAccBufs
      if (!mbar_wait(&acc_empty[a], ((li / kAccBufs) & 1u) ^ 1u, abort_flag, p.err_word, p.timeout_ns)) {
        ok = false;
        break;
      }
      MetaSlot<NB>& m = meta[a];
      m.pt[t] = cur.pt;
      m.np[t] = cur.np;
      m.sp[t] = cur.sp;
      if (t < NB) {
        m.lid[t] = cur.lid;
        m.lg[t] = cur.lg;
        m.lnls[(t >> 1) * 4u + (t & 1u)] = cur.ln;
        m.lnls[(t >> 1) * 4u + 2u + (t & 1u)] = cur.ls;
      }
      if (t == 0) {
        m.task = cur.task;
        m.rh = cur.rh;
        m.nl = cur.nl;
        m.r0 = cur.r0;
        m.tout = cur.tout;
      }
      mbar_arrive(&meta_full[a]);
      for (uint32_t sl = 0; sl < nslab; ++sl) {
        if (has_next && sl < 4) prod_step<NB>(p, next, sl, nxt, t);
        const uint32_t st = gs % S;
        if (!mbar_wait(&empty[st], ((gs / S) & 1u) ^ 1u, abort_flag, p.err_word, p.timeout_ns)) {
          ok = false;
          break;
        }
        const uint32_t off = sl * kSlabTc + piece * 16u;
        const uint32_t n = off < pd ? 16u : 0u;
        const uint32_t adst = ring0 + st * G::kStage + row0 * kSlabTc + swz;
#pragma unroll
        for (uint32_t u = 0; u < 8; ++u) {
          const uint32_t nu = cur.crow[u] != 0xffffffffu ? n : 0u;
          cp_async16(adst + u * 16u * kSlabTc, nu ? p.codes + (uint64_t)cur.crow[u] * pd + off : p.codes, nu);
        }
        const uint32_t bdst = ring0 + st * G::kStage + kASlabTc + row0 * kSlabTc + swz;
#pragma unroll
        for (uint32_t v = 0; v < NB / 16u; ++v) {
          const uint32_t nv = cur.lrow[v] != 0xffffffffu ? n : 0u;
          cp_async16(bdst + v * 16u * kSlabTc, nv ? p.codes + (uint64_t)cur.lrow[v] * pd + off : p.codes, nv);
        }
        cp_async_mbar_arrive(&full[st]);
        ++gs;
      }
      if (has_next)
        for (uint32_t step = nslab; step < 4; ++step) prod_step<NB>(p, next, step, nxt, t);
      cur = nxt;
    }
    cp_async_wait_all();  // nothing in flight when the CTA leaves
  } else if (warp < kMmaWarp) {
    // ------------------------------------------------------------ epilogue
    // group a takes items a, a + kAccBufs, ... of this CTA (accumulator buffer
    // and metadata slot a); warp 4 + 4a + q reads TMEM lane quadrant q.
    const uint32_t a = (warp - kEpiWarp0) >> 2, q = warp & 3u;
    const uint32_t row = q * 32u + lane;
    for (uint32_t item = blockIdx.x + a * gridDim.x, li = a; item < p.num_work;
         item += kAccBufs * gridDim.x, li += kAccBufs) {
      const uint32_t ph = (li / kAccBufs) & 1u;
      bool ok = true;
      if (lane == 0)
        ok = mbar_wait(&meta_full[a], ph, abort_flag, p.err_word, p.timeout_ns) &&
             mbar_wait(&acc_full[a], ph, abort_flag, p.err_word, p.timeout_ns);
      if (__shfl_sync(0xffffffffu, ok ? 1u : 0u, 0) == 0u) break;
      tc_fence_after();
      const MetaSlot<NB>& m = meta[a];
      const uint32_t point = m.pt[row], nl = m.nl, rh = m.rh;
      const bool valid = point != 0xffffffffu;
      const float n_p = m.np[row], s_p = m.sp[row];
      float bd[4];
      uint32_t bs[4], bl[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        bd[j] = 3.402823466e+38F;
        bs[j] = 0xffffffffu;
        bl[j] = 0xffffffffu;
      }
      // Reject bound: a candidate more than the 2e-5 tie window above it is
      // neither better than nor tied with any slot the insertion would compare
      // it to (CB:6524-6578), so it cannot enter.  Slot mode compares with its
      // last slot first; the four-slot list with every slot (the maximum).
      //
      // Per 16 leaders: the distances two at a time on register pairs (paired
      // f32 instructions round each element as the scalar form; -2 s_p l_s is
      // exact negation of the reference's 2 s_p l_s), and a mask of the
      // leaders not rejected against the bound at the block's start.  The
      // bound only falls and clamping only raises a distance, so a leader
      // outside the mask is rejected in the sequential order too; the masked
      // ones are taken in ascending slot order and get the exact sequential
      // test (clamped distance, current bound) before the insertion.
      float worst = 3.402823466e+38F;
      const float nsp = -2.0f * s_p;
      const uint64_t np2 = f2_pack(n_p, n_p), nsp2 = f2_pack(nsp, nsp);
      const float4* lm4 = reinterpret_cast<const float4*>(m.lnls);
#pragma unroll 1
      for (uint32_t c0 = 0; c0 < NB; c0 += 16) {
        uint32_t v[16];
        tmem_ld_32x32b_x16(tmem_base + ((q * 32u) << 16) + a * NB + c0, v);
        tmem_ld_wait();
        if (valid) {
          float d[16];
          uint32_t mask = 0u;
          const uint64_t nw2 = f2_pack(-worst, -worst);
#pragma unroll
          for (uint32_t j = 0; j < 16; j += 2) {
            const float4 lm = lm4[(c0 + j) >> 1];  // ln_l, ln_l+1, ls_l, ls_l+1
            const uint64_t nn = f2_add(np2, f2_pack(lm.x, lm.y));
            const uint64_t ntt = f2_mul(nsp2, f2_pack(lm.z, lm.w));
            const uint64_t df = f2_pack(__int2float_rn((int)v[j]), __int2float_rn((int)v[j + 1]));
            const uint64_t dd = p.fused ? f2_fma(ntt, df, nn) : f2_add(nn, f2_mul(ntt, df));
            f2_unpack(dd, d[j], d[j + 1]);
            float r0, r1;
            f2_unpack(f2_add(dd, nw2), r0, r1);  // rn(d - worst)
            mask |= (!(r0 > 2.0e-5f) ? 1u : 0u) << j;
            mask |= (!(r1 > 2.0e-5f) ? 1u : 0u) << (j + 1u);
          }
          while (mask != 0u) {
            const uint32_t j = __ffs(mask) - 1u;
            mask &= mask - 1u;
            const uint32_t l = c0 + j;
            float dj = select16(d, j);
            if (dj <= 0.0f) dj = 0.0f;
            const uint32_t lid = m.lid[l];
            if (lid == 0xffffffffu || __fsub_rn(dj, worst) > 2.0e-5f) continue;
            if constexpr (SLOTS) {
              insertn(dj, point, lid, l, rh, bd, bs, bl);
              worst = rh == 1u ? bd[0] : (rh == 2u ? bd[1] : (rh == 3u ? bd[2] : bd[3]));
            } else {
              insert4(dj, point, lid, l, bd, bs, bl);
              worst = fmaxf(fmaxf(bd[0], bd[1]), fmaxf(bd[2], bd[3]));
            }
          }
        }
      }
      if (valid) {
        const uint64_t out = m.tout + (uint64_t)(m.r0 + row) * rh;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if ((uint32_t)j >= rh) break;
          if (bs[j] >= nl) {
            atomicOr(p.err_word, TESSA_DEVERR_BAD_TASK);
            continue;
          }
          if constexpr (SLOTS) {
            p.out_slots[out + j] = bs[j];
            if (p.out_dists) p.out_dists[out + j] = bd[j];
          } else {
            p.out_ids[out + j] = m.lg[bs[j]];
            p.out_dists[out + j] = bd[j];
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[a]);
    }
  } else if (lane == 0) {
    // ------------------------------------------------------------ MMA issuer
    const uint32_t idesc = idesc_i8(kRowsTc, NB);
    uint32_t gs = 0;
    bool ok = true;
    for (uint32_t item = blockIdx.x, li = 0; ok && item < p.num_work; item += gridDim.x, ++li) {
      const uint32_t a = li % kAccBufs;
      if (!mbar_wait(&acc_empty[a], ((li / kAccBufs) & 1u) ^ 1u, abort_flag, p.err_word, p.timeout_ns)) break;
      tc_fence_after();
      for (uint32_t sl = 0; sl < nslab; ++sl, ++gs) {
        const uint32_t st = gs % S;
        if (!mbar_wait(&full[st], (gs / S) & 1u, abort_flag, p.err_word, p.timeout_ns)) {
          ok = false;
          break;
        }
        // the stage's copies have landed: the barrier completes only after
        // every producer's cp.async writes are done
        tc_fence_after();
        const uint32_t aa = ring0 + st * G::kStage, ba = aa + kASlabTc;
#pragma unroll
        for (uint32_t kk = 0; kk < kSlabTc / kMmaKTc; ++kk)
          mma_i8_ss(tmem_base + a * NB, smem_desc_sw128(aa + kk * kMmaKTc), smem_desc_sw128(ba + kk * kMmaKTc),
                    idesc, (sl | kk) != 0u ? 1u : 0u);
        mma_commit(&empty[st]);
        if (sl + 1 == nslab) mma_commit(&acc_full[a]);
      }
    }
    // every issued MMA has landed before TMEM is released
    mma_commit(done_bar);
    uint32_t dummy_abort = 0u;
    mbar_wait(done_bar, 0u, &dummy_abort, p.err_word, p.timeout_ns);
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem_base, G::kTmemCols);
  }
}

template <uint32_t NB, bool SLOTS>
static int launch_nb_mode(const Params& prm, int sm_count, cudaStream_t stream) {
  const uint32_t smem = Geom<NB>::kSmem;
  if (cudaFuncSetAttribute(assign_tc_kernel<NB, SLOTS>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
      cudaSuccess)
    return TESSA_ERR_CUDA;
  const uint32_t cap = (uint32_t)sm_count;  // one CTA per SM
  const uint32_t grid = prm.num_work < cap ? prm.num_work : cap;
  assign_tc_kernel<NB, SLOTS><<<grid, kThreadsTc, smem, stream>>>(prm);
  return cudaGetLastError() == cudaSuccess ? TESSA_OK : TESSA_ERR_CUDA;
}

template <uint32_t NB>
static int launch_nb(const Params& prm, int sm_count, cudaStream_t stream) {
  return prm.out_slots ? launch_nb_mode<NB, true>(prm, sm_count, stream)
                       : launch_nb_mode<NB, false>(prm, sm_count, stream);
}

}  // namespace tc
}  // namespace assign

// SQ8 assignment on the tensor cores when every task has at most 128 leaders;
// TESSA_ERR_UNSUPPORTED otherwise (the caller then runs the SIMT kernel).
int launch_assign_sq8_tc(const assign::Params& prm, uint32_t max_leaders, int sm_count, cudaStream_t stream) {
  if (prm.num_work == 0) return TESSA_OK;
  if (max_leaders == 0 || max_leaders > assign::tc::kMaxNB) return TESSA_ERR_UNSUPPORTED;
  if (max_leaders <= 16) return assign::tc::launch_nb<16>(prm, sm_count, stream);
  if (max_leaders <= 32) return assign::tc::launch_nb<32>(prm, sm_count, stream);
  if (max_leaders <= 64) return assign::tc::launch_nb<64>(prm, sm_count, stream);
  return assign::tc::launch_nb<128>(prm, sm_count, stream);
}

}  // namespace tessa
