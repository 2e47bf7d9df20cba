// Cross-depth masked flash attention backward, dK / dV half (tcgen05), as a
// persistent kernel: the backward of reference src/pe/nn.py:84-88 under the
// mask of src/pe/masks.py:43-61, partition slot layout (src/pe/partition.py:41-55).
//
// Work item = (query head h, 128-key tile) for key tiles many queries read, and
// (KV head, 128-key tile) -- all rep query heads of the group in turn, dK / dV
// summed in TMEM -- for the light tiles of prediction-slot keys (each read by
// the two 64-query steps of its own anchors).  One CTA per SM takes items from
// a global counter in order of decreasing work (key tiles ascending, heads
// fastest; the grouped light tiles last), so TMEM allocation, barrier set-up
// and the first loads happen once per CTA and the next item's K / V / Q / dO
// loads overlap the current item.
// For an item it walks, in 64-query steps, the query rows that can read the key
// tile (keys on TMEM lanes):
//   S^T  = K Q^T           dP^T = V dO^T           (N = 64)
//   P^T  = 2^(S^T c - lse')  dS^T = P^T (dP^T - delta)   (compute warps; bf16
//          packed back over S^T / dP^T; masked pairs exactly zero)
//   dV  += P^T dO           dK  += dS^T Q
// Both score tiles are double-buffered in TMEM and issued together two steps
// ahead: per step the MMAs issue as
//   dV(i), dK(i), S^T(i+2), dP^T(i+2)
// once every compute warp has written P^T(i) and dS^T(i), so a compute warp's
// step is one wait, one pair of TMEM loads and one pair of stores, and step
// i + 1 (whose scores are in since step i - 1) overlaps the MMAs of step i.
// dV and dK take A from TMEM (P^T / dS^T written by the
// compute warps, 64 B of shared memory per clock for B); S^T = K Q^T and
// dP^T = V dO^T keep both operands in shared memory (an M = 128, N = 64 MMA
// then runs at ~2/3 rate on shared-memory bandwidth), which leaves TMEM room
// for the second dP^T buffer.
// The item's dK / dV tile is added (fp32) into the KV head's accumulators,
// reducing the query heads of a GQA group without expanding K / V.
//
// Warp roles (640 threads):
//   warp 0      scheduler + TMA: claims items; K per item (two buffers), V per
//               item (one buffer, refilled once the item's last dP^T read it);
//               Q / dO per step into 4- and 3-deep rings
//   warp 1      tcgen05.mma issue
//   warp 2      per-query operands (lse * log2 e, delta, anchor, depth) per step
//   warp 3      idle
//   warps 4-19  compute: four per TMEM lane quarter, each owning 16 of the 64
//               query columns; parts 0 / 1 drain the two halves of the previous
//               item's dK, parts 2 / 3 of its dV, before the item's first P^T
// TMEM: dK 0..127, dV 128..255, S^T 256..319 / 320..383, dP^T 384..447 /
//       448..511.
#include "attn_tc.cuh"

namespace pe {
namespace {

using namespace sm100;
using namespace attn_tc;

constexpr int QT = 64;                          // queries per step
constexpr uint32_t SUB_BYTES = QT * HD * 2;      // 16 KB: 64 rows x 128 bf16
constexpr uint32_t SUB_CHUNK = SUB_BYTES / 2;    // 8 KB: 64 rows x 128 B
constexpr int QS = 4, DS = 3, MS = 4;           // ring depths: Q, dO, per-query operands
constexpr int kComputeWarps = 16;               // four per TMEM lane quarter
constexpr int kThreads = 128 + 32 * kComputeWarps;
constexpr int kParts = kComputeWarps / 4;
constexpr int kCols = QT / kParts;              // query columns per compute warp
constexpr int kGroupSteps = 32;                 // a key tile with at most this many steps over
                                                // a GQA group runs as one item per KV head

// shared memory (offsets from the 1024-aligned base)
constexpr uint32_t OFF_K = 0;                        // [2] K tiles
constexpr uint32_t OFF_V = OFF_K + 2 * TILE_BYTES;
constexpr uint32_t OFF_Q = OFF_V + TILE_BYTES;
constexpr uint32_t OFF_DO = OFF_Q + QS * SUB_BYTES;
constexpr uint32_t OFF_L = OFF_DO + DS * SUB_BYTES;   // float [MS][QT]  -lse * log2 e
constexpr uint32_t OFF_D = OFF_L + MS * QT * 4;       // float [MS][QT]  -delta
constexpr uint32_t OFF_A = OFF_D + MS * QT * 4;       // int   [MS][QT]  anchor (-1: no row)
constexpr uint32_t OFF_E = OFF_A + MS * QT * 4;       // int   [MS][QT]  depth
constexpr uint32_t OFF_ITEM = OFF_E + MS * QT * 4;    // int   [2]
constexpr uint32_t OFF_BAR = OFF_ITEM + 16;
constexpr int NBARS = 2 + 2 + 2 + 2 + 1 + 1 + 2 * QS + 2 * DS + 2 * MS + 2 + 2 + 2 + 1;
constexpr uint32_t OFF_TMEM = OFF_BAR + NBARS * 8;
constexpr size_t SMEM_KV2 = 1024 + OFF_TMEM + 16;

struct Bars {
  uint64_t *item_full, *item_empty, *k_full, *k_empty, *v_full, *v_empty, *q_full, *q_empty,
      *do_full, *do_empty, *meta_full, *meta_empty, *st_full, *dpt_full, *ds_full,
      *acc_full;
  __device__ explicit Bars(uint64_t* b) {
    item_full = b; b += 2;
    item_empty = b; b += 2;
    k_full = b; b += 2;      // K tile (per item parity) landed
    k_empty = b; b += 2;     // the item's last S^T read it
    v_full = b; b += 1;      // V tile landed in shared memory
    v_empty = b; b += 1;     // the item's last dP^T read it
    q_full = b; b += QS;
    q_empty = b; b += QS;
    do_full = b; b += DS;
    do_empty = b; b += DS;
    meta_full = b; b += MS;
    meta_empty = b; b += MS;
    st_full = b; b += 2;     // per score buffer: S^T landed
    dpt_full = b; b += 2;    // per score buffer: dP^T landed
    ds_full = b; b += 2;     // per score buffer: P^T and dS^T written back
    acc_full = b; b += 1;
  }
};

// Items: the first tab.nsplit units (key tiles) run as Hq items, one per query
// head; every later unit as Hkv items, one per KV head walking all rep query
// heads of its group, so a key tile few queries read pays the item's fixed cost
// (K / V load, pipeline fill, dK / dV drain) once per group instead of per head.
__device__ __forceinline__ int item_total(const SegTable& tab, int Hq, int Hkv) {
  const int units = tab.nwork > 0 ? tab.nwork : (tab.g[0].S + TK - 1) / TK;
  return Hq * tab.nsplit + Hkv * (units - tab.nsplit);
}

// the item's segment, key tile, query heads and the 64-query steps that read it
struct Item {
  int seg, h0, nh, kvh, k0;
  PartGeom g;
  int64_t ml;  // first lse / delta element of the segment: Hq * its first stacked row
  int64_t r0;  // its first stacked row
  Ranges qr;
  int nq;      // 64-query steps per query head
  int n;       // steps of the item: nq for each of its nh heads, head-major
  __device__ Item(int w, int Hq, int Hkv, int rep, const SegTable& tab) {
    const int head_items = Hq * tab.nsplit;
    int e;
    if (w < head_items) {
      e = w / Hq;
      h0 = w - e * Hq;
      nh = 1;
      kvh = h0 / rep;
    } else {
      const int r = w - head_items;
      e = r / Hkv;
      kvh = r - e * Hkv;
      e += tab.nsplit;
      h0 = kvh * rep;
      nh = rep;
    }
    int kt;
    if (tab.nwork > 0) {
      unpack_work(tab.work[e], seg, kt);
    } else {
      seg = 0;
      kt = e;
    }
    g = tab.g[seg];
    r0 = tab.row0[seg];
    ml = (int64_t)Hq * r0;
    k0 = kt * TK;
    qr = query_tiles(g, k0, QT);
    nq = qr.count();
    n = nq * nh;
  }
  // query head and 64-query tile of step i
  __device__ __forceinline__ int head(int i) const { return nh > 1 ? h0 + i / nq : h0; }
  __device__ __forceinline__ int qtile(int i) const { return qr.at(nh > 1 ? i % nq : i); }
};

// packed P^T / dS^T: the queries of compute part p (columns [p C, p C + C)) sit in
// columns [p C, p C + C / 2) of their tile, which only part p writes
__device__ __forceinline__ uint32_t a_col(int kk) {
  constexpr int steps = kCols / 16;
  return (uint32_t)((kk / steps) * kCols + (kk % steps) * 8);
}

__global__ void __launch_bounds__(kThreads, 1)
attn_bwd_kv2_kernel(const __grid_constant__ SegTable tab, const float* __restrict__ lse,
                    const float* __restrict__ delta, float* __restrict__ dk_acc,
                    float* __restrict__ dv_acc, int* work_counter, int Hq, int Hkv, int rep,
                    float scale, int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sK = smem + OFF_K;
  uint8_t* sV = smem + OFF_V;
  float* sL = reinterpret_cast<float*>(smem + OFF_L);
  float* sD = reinterpret_cast<float*>(smem + OFF_D);
  int* sA = reinterpret_cast<int*>(smem + OFF_A);
  int* sE = reinterpret_cast<int*>(smem + OFF_E);
  volatile int* sItem = reinterpret_cast<volatile int*>(smem + OFF_ITEM);
  Bars B(reinterpret_cast<uint64_t*>(smem + OFF_BAR));
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_TMEM);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // items: (work-list entry or, for a lone segment, key tile) x query head
  const int total = item_total(tab, Hq, Hkv);

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&B.item_full[i], 1);
      mbar_init(&B.item_empty[i], 2 + kComputeWarps);  // MMA, operands, compute warps
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&B.k_full[i], 1);
      mbar_init(&B.k_empty[i], 1);
      mbar_init(&B.st_full[i], 1);
    }
    mbar_init(B.v_full, 1);
    mbar_init(B.v_empty, 1);
    for (int i = 0; i < QS; ++i) {
      mbar_init(&B.q_full[i], 1);
      mbar_init(&B.q_empty[i], 1);
    }
    for (int i = 0; i < DS; ++i) {
      mbar_init(&B.do_full[i], 1);
      mbar_init(&B.do_empty[i], 1);
    }
    for (int i = 0; i < MS; ++i) {
      mbar_init(&B.meta_full[i], 32);
      mbar_init(&B.meta_empty[i], kComputeWarps);
    }
    // the scores run two steps ahead, so a fast warp may reach step i + 1 before a
    // slow one arrives for step i (never step i + 2): one barrier set per buffer
    for (int i = 0; i < 2; ++i) {
      mbar_init(&B.dpt_full[i], 1);
      mbar_init(&B.ds_full[i], kComputeWarps);
    }
    mbar_init(B.acc_full, 1);
    fence_barrier_init();
    fence_proxy_async();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tDK = tmem, tDV = tmem + 128;
  const uint32_t tS = tmem + 256, tDP = tmem + 384;  // buffer b at + b * QT

  // every role walks the same item sequence; `ic` counts items, `gs` steps
  auto read_item = [&](int ic, bool& ok) -> int {
    if (!mbar_wait(&B.item_full[ic & 1], (ic >> 1) & 1, status, 340)) {
      ok = false;
      return -1;
    }
    const int w = sItem[ic & 1];
    __syncwarp();
    if (lane == 0) mbar_arrive(&B.item_empty[ic & 1]);
    return w;
  };

  if (warp == 0) {
    // ---------------- scheduler + TMA ----------------
    if (elect_one()) {
      bool ok = true;
      uint64_t* last_bar = nullptr;
      uint32_t last_ph = 0;
      int gs = 0;
      for (int ic = 0;; ++ic) {
        int w = atomicAdd(work_counter, 1);
        if (w >= total) w = -1;
        if (!mbar_wait(&B.item_empty[ic & 1], ((ic >> 1) & 1) ^ 1u, status, 341)) { ok = false; break; }
        sItem[ic & 1] = w;
        mbar_arrive(&B.item_full[ic & 1]);  // release: publishes the slot write
        if (w < 0) break;
        const Item it(w, Hq, Hkv, rep, tab);
        // K into buffer ic & 1 once the item two back issued its last S^T
        const int kb = ic & 1;
        if (!mbar_wait(&B.k_empty[kb], ((ic >> 1) & 1) ^ 1u, status, 342)) { ok = false; break; }
        uint8_t* kd = sK + kb * TILE_BYTES;
        mbar_arrive_expect_tx(&B.k_full[kb], TILE_BYTES);
        tma_load_2d(kd, &tab.tm[it.seg][1], &B.k_full[kb], it.kvh * HD, it.k0);
        tma_load_2d(kd + CHUNK, &tab.tm[it.seg][1], &B.k_full[kb], it.kvh * HD + 64, it.k0);
        last_bar = &B.k_full[kb];
        last_ph = (ic >> 1) & 1;
        // V once the previous item's last dP^T read it
        if (!mbar_wait(B.v_empty, (ic & 1) ^ 1u, status, 357)) { ok = false; break; }
        mbar_arrive_expect_tx(B.v_full, TILE_BYTES);
        tma_load_2d(sV, &tab.tm[it.seg][2], B.v_full, it.kvh * HD, it.k0);
        tma_load_2d(sV + CHUNK, &tab.tm[it.seg][2], B.v_full, it.kvh * HD + 64, it.k0);
        last_bar = B.v_full;
        last_ph = ic & 1;
        for (int i = 0; i < it.n && ok; ++i) {
          const int gi = gs + i;
          const int q0 = it.qtile(i) * QT, hc = it.head(i) * HD;
          const int qs = gi % QS, ds = gi % DS;
          if (!mbar_wait(&B.q_empty[qs], ((gi / QS) & 1) ^ 1u, status, 343)) { ok = false; break; }
          uint8_t* qd = smem + OFF_Q + qs * SUB_BYTES;
          mbar_arrive_expect_tx(&B.q_full[qs], SUB_BYTES);
          tma_load_2d(qd, &tab.tm[it.seg][0], &B.q_full[qs], hc, q0);
          tma_load_2d(qd + SUB_CHUNK, &tab.tm[it.seg][0], &B.q_full[qs], hc + 64, q0);
          last_bar = &B.q_full[qs];
          last_ph = (gi / QS) & 1;
          if (!mbar_wait(&B.do_empty[ds], ((gi / DS) & 1) ^ 1u, status, 344)) { ok = false; break; }
          uint8_t* dd = smem + OFF_DO + ds * SUB_BYTES;
          mbar_arrive_expect_tx(&B.do_full[ds], SUB_BYTES);
          tma_load_2d(dd, &tab.tm[it.seg][3], &B.do_full[ds], hc, q0);
          tma_load_2d(dd + SUB_CHUNK, &tab.tm[it.seg][3], &B.do_full[ds], hc + 64, q0);
          last_bar = &B.do_full[ds];
          last_ph = (gi / DS) & 1;
        }
        if (!ok) break;
        gs += it.n;
      }
      // on a failed wait, let this thread's last copy land before the CTA exits
      if (!ok && last_bar) mbar_wait(last_bar, last_ph, nullptr, 0);
    }
  } else if (warp == 1) {
    // ---------------- MMA issue ----------------
    bool ok = true;
    int gs = 0;
    constexpr uint32_t ID_KQ = idesc_bf16(TK, QT, false, false);  // S^T, dP^T
    constexpr uint32_t ID_KM = idesc_bf16(TK, HD, false, true);   // dV, dK (A = P^T / dS^T)
    for (int ic = 0; ok; ++ic) {
      const int w = read_item(ic, ok);
      if (w < 0) break;
      const bool leader = elect_one();
      const int leader_lane = __ffs(__ballot_sync(0xffffffffu, leader)) - 1;
      if (leader) {
        const Item it(w, Hq, Hkv, rep, tab);
        const int kb = ic & 1, last = gs + it.n - 1;
        const uint32_t k_base = smem_u32(sK + kb * TILE_BYTES);
        // S^T(gi) = K Q(gi)^T into buffer gi & 1, both operands in shared memory
        auto issue_st = [&](int gi) -> bool {
          const int qs = gi % QS;
          if (!mbar_wait(&B.q_full[qs], (gi / QS) & 1, status, 345)) return false;
          tc_fence_after();
          const uint32_t q_base = smem_u32(smem + OFF_Q + qs * SUB_BYTES);
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk)
            mma_bf16_ss(tS + (gi & 1) * QT,
                        sw128_desc(k_base + (kk >> 2) * CHUNK + (kk & 3) * 32, 16, 1024),
                        sw128_desc(q_base + (kk >> 2) * SUB_CHUNK + (kk & 3) * 32, 16, 1024),
                        ID_KQ, kk > 0 ? 1u : 0u);
          mma_commit(&B.st_full[gi & 1]);
          if (gi == last) mma_commit(&B.k_empty[kb]);  // the item's last read of K
          return true;
        };
        // dP^T(gi) = V dO(gi)^T into buffer gi & 1, both operands in shared memory
        const uint32_t v_base = smem_u32(sV);
        auto issue_dpt = [&](int gi) -> bool {
          const int ds = gi % DS;
          if (!mbar_wait(&B.do_full[ds], (gi / DS) & 1, status, 346)) return false;
          tc_fence_after();
          const uint32_t do_base = smem_u32(smem + OFF_DO + ds * SUB_BYTES);
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk)
            mma_bf16_ss(tDP + (gi & 1) * QT,
                        sw128_desc(v_base + (kk >> 2) * CHUNK + (kk & 3) * 32, 16, 1024),
                        sw128_desc(do_base + (kk >> 2) * SUB_CHUNK + (kk & 3) * 32, 16, 1024),
                        ID_KQ, kk > 0 ? 1u : 0u);
          mma_commit(&B.dpt_full[gi & 1]);
          if (gi == last) mma_commit(B.v_empty);  // the item's last read of V
          return true;
        };
        ok = mbar_wait(&B.k_full[kb], (ic >> 1) & 1, status, 347);
        if (ok && it.n == 0) {
          // nothing reads this key tile: release K and V without MMAs
          mma_commit(&B.k_empty[kb]);
          ok = mbar_wait(B.v_full, ic & 1, status, 358);
          if (ok) mma_commit(B.v_empty);
        }
        if (ok && it.n > 0) {
          tc_fence_after();
          ok = issue_st(gs);
        }
        if (ok && it.n > 1) ok = issue_st(gs + 1);
        if (ok && it.n > 0) ok = mbar_wait(B.v_full, ic & 1, status, 358);
        if (ok && it.n > 0) {
          tc_fence_after();
          ok = issue_dpt(gs);
        }
        if (ok && it.n > 1) ok = issue_dpt(gs + 1);
        for (int i = 0; i < it.n && ok; ++i) {
          const int gi = gs + i, b = gi & 1;
          const uint32_t acc = i > 0 ? 1u : 0u;
          // P^T(i) and dS^T(i) written by every compute warp
          if (!mbar_wait(&B.ds_full[b], (gi >> 1) & 1, status, 348)) { ok = false; break; }
          tc_fence_after();
          const uint32_t do_base = smem_u32(smem + OFF_DO + (gi % DS) * SUB_BYTES);
#pragma unroll
          for (int kk = 0; kk < QT / 16; ++kk)
            mma_bf16_ts(tDV, tS + b * QT + a_col(kk),
                        sw128_desc(do_base + kk * 2048, SUB_CHUNK, 1024), ID_KM,
                        (acc | kk) != 0 ? 1u : 0u);
          mma_commit(&B.do_empty[gi % DS]);  // dO(gi): dP^T(gi) and dV(gi) issued
          const uint32_t q_base = smem_u32(smem + OFF_Q + (gi % QS) * SUB_BYTES);
#pragma unroll
          for (int kk = 0; kk < QT / 16; ++kk)
            mma_bf16_ts(tDK, tDP + b * QT + a_col(kk),
                        sw128_desc(q_base + kk * 2048, SUB_CHUNK, 1024), ID_KM,
                        (acc | kk) != 0 ? 1u : 0u);
          mma_commit(&B.q_empty[gi % QS]);  // Q(gi): S^T(gi) and dK(gi) issued
          // S^T(i+2) / dP^T(i+2) overwrite P^T(i) / dS^T(i) after dV(i) / dK(i) read
          // them (tcgen05 executes in issue order)
          if (i + 2 < it.n && !issue_st(gi + 2)) { ok = false; break; }
          if (i + 2 < it.n && !issue_dpt(gi + 2)) { ok = false; break; }
        }
        if (ok) mma_commit(B.acc_full);
        gs += it.n;
      }
      __syncwarp();
      ok = __shfl_sync(0xffffffffu, ok, leader_lane);
      gs = __shfl_sync(0xffffffffu, gs, leader_lane);
    }
  } else if (warp == 2) {
    // ---------------- per-query operands ----------------
    bool ok = true;
    int gs = 0;
    for (int ic = 0; ok; ++ic) {
      const int w = read_item(ic, ok);
      if (w < 0) break;
      const Item it(w, Hq, Hkv, rep, tab);
      for (int i = 0; i < it.n; ++i) {
        const int gi = gs + i, slot = gi % MS;
        const int q0 = it.qtile(i) * QT;
        const int64_t hrow = it.ml + (int64_t)it.head(i) * it.g.S;
        if (!mbar_wait(&B.meta_empty[slot], ((gi / MS) & 1) ^ 1u, status, 350)) ok = false;
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
#pragma unroll
        for (int u = 0; u < QT / 32; ++u) {
          const int r = u * 32 + lane, q = q0 + r;
          // staged negated, so the compute warps add them with packed f32x2 ops
          float lv = -INFINITY, dl = 0.f;
          int qa = -1, qd = 0;
          if (q < it.g.S) {
            lv = -lse[hrow + q] * kLog2e;
            dl = -delta[hrow + q];
            decode(it.g, q, qa, qd);
          }
          sL[slot * QT + r] = lv;
          sD[slot * QT + r] = dl;
          sA[slot * QT + r] = qa;
          sE[slot * QT + r] = qd;
        }
        mbar_arrive(&B.meta_full[slot]);  // every lane: release of its own writes
      }
      gs += it.n;
    }
  } else if (warp >= 4) {
    // ---------------- compute: thread = key row (TMEM lane) ----------------
    constexpr int C = kCols;
    const int quarter = warp & 3;
    const int part = (warp - 4) >> 2;
    const int cb = part * C;
    const int row = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const float scale_log2 = scale * kLog2e;
    const float2 sc2 = make_float2(scale_log2, scale_log2);
    const int64_t kv_ld = (int64_t)Hkv * HD;
    bool ok = true;
    int gs = 0;
    // the previous item's dK (parts 0, 1) / dV (parts 2, 3) row, drained before this
    // item's first P^T: the item's first dV / dK MMAs (which overwrite the
    // accumulators) wait for that P^T, while its first S^T / dP^T already run
    float* pending = nullptr;
    bool have_pending = false;
    auto drain = [&](int ic_prev) -> bool {
      if (!mbar_wait(B.acc_full, ic_prev & 1, status, 354)) return false;
      tc_fence_after();
      const int half = (part & 1) * (HD / 2);
      const uint32_t src = (part < 2 ? tDK : tDV) + lane_off + half;
#pragma unroll 1
      for (int c0 = 0; c0 < HD / 2; c0 += 32) {
        float v[32];
        tmem_ld32(src + c0, v);
        tmem_wait_ld();
        if (pending) atomic_add_row32(pending + half + c0, v, 1.f);
      }
      return true;
    };
    int ic = 0;
    for (; ok; ++ic) {
      const int w = read_item(ic, ok);
      if (w < 0) break;
      const Item it(w, Hq, Hkv, rep, tab);
      const int kj = it.k0 + row;
      const bool kvalid = kj < it.g.S;
      int ka = 0, ke = 0;
      if (kvalid) decode(it.g, kj, ka, ke);
      if (have_pending && !drain(ic - 1)) { ok = false; break; }
      // (an item no query reads leaves the accumulators untouched: nothing to add)
      pending = kvalid && it.n > 0
                    ? (part < 2 ? dk_acc : dv_acc) + (it.r0 + kj) * kv_ld + it.kvh * HD
                    : nullptr;
      have_pending = true;
      for (int i = 0; i < it.n; ++i) {
        const int gi = gs + i, slot = gi % MS, b = gi & 1;
        const int q0 = it.qtile(i) * QT;
        const bool full = tile_fully_allowed(it.g, q0, it.k0, QT);
        // ---- P^T = 2^(S^T c - lse') and dS^T = P^T (dP^T - delta): S^T(i) and
        // dP^T(i) were issued together two steps ahead, so one wait, one pair of TMEM
        // loads and one pair of stores cover the step ----
        if (!mbar_wait(&B.meta_full[slot], (gi / MS) & 1, status, 351)) { ok = false; break; }
        if (!mbar_wait(&B.st_full[b], (gi >> 1) & 1, status, 352)) { ok = false; break; }
        if (!mbar_wait(&B.dpt_full[b], (gi >> 1) & 1, status, 353)) { ok = false; break; }
        tc_fence_after();
        float pv[C], dv[C];
        tmem_ld16(tS + b * QT + lane_off + cb, pv);
        tmem_ld16(tDP + b * QT + lane_off + cb, dv);
        tmem_wait_ld();
        const float* L = sL + slot * QT + cb;
        if (full) {
#pragma unroll
          for (int c = 0; c < C; c += 4) {
            const float4 l4 = *reinterpret_cast<const float4*>(L + c);
            const float2 e0 = fma2(make_float2(pv[c], pv[c + 1]), sc2, make_float2(l4.x, l4.y));
            const float2 e1 =
                fma2(make_float2(pv[c + 2], pv[c + 3]), sc2, make_float2(l4.z, l4.w));
            pv[c] = ex2_approx(e0.x);
            pv[c + 1] = ex2_approx(e0.y);
            pv[c + 2] = ex2_approx(e1.x);
            pv[c + 3] = ex2_approx(e1.y);
          }
        } else {
          const int* QA = sA + slot * QT + cb;
          const int* QE = sE + slot * QT + cb;
#pragma unroll
          for (int c = 0; c < C; ++c) {
            const int qa = QA[c];
            const bool allow =
                kvalid && qa >= 0 && (ke == 0 ? (ka <= qa) : (ka == qa && ke <= QE[c]));
            pv[c] = allow ? ex2_approx(fmaf(pv[c], scale_log2, L[c])) : 0.f;
          }
        }
        const float* D = sD + slot * QT + cb;
        uint32_t pw[C / 2], sw[C / 2];
#pragma unroll
        for (int c = 0; c < C; c += 4) {
          const float4 d4 = *reinterpret_cast<const float4*>(D + c);
          const float2 s0 = mul2(make_float2(pv[c], pv[c + 1]),
                                 add2(make_float2(dv[c], dv[c + 1]), make_float2(d4.x, d4.y)));
          const float2 s1 = mul2(make_float2(pv[c + 2], pv[c + 3]),
                                 add2(make_float2(dv[c + 2], dv[c + 3]), make_float2(d4.z, d4.w)));
          pw[c / 2] = pack_bf16x2(pv[c], pv[c + 1]);
          pw[c / 2 + 1] = pack_bf16x2(pv[c + 2], pv[c + 3]);
          sw[c / 2] = pack_bf16x2(s0.x, s0.y);
          sw[c / 2 + 1] = pack_bf16x2(s1.x, s1.y);
        }
        tmem_st8(tS + b * QT + lane_off + cb, pw);
        tmem_st8(tDP + b * QT + lane_off + cb, sw);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&B.ds_full[b]);
          mbar_arrive(&B.meta_empty[slot]);
        }
      }
      if (!ok) break;
      gs += it.n;
    }
    // the last item's dK / dV
    if (ok && have_pending) drain(ic - 1);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

int attn_bwd_kv2_launch(int nseg, const PartGeom* g, int Hq, int Hkv, const void* q,
                        int64_t q_ss, const void* k, int64_t k_ss, const void* v, int64_t v_ss,
                        const void* dout, int64_t do_ss, const float* lse, const float* delta,
                        float* dk_acc, float* dv_acc, int* work_counter, int* status,
                        cudaStream_t st) {
  PE_CHECK_ARG(nseg >= 1 && nseg <= kMaxSeg, "attention backward: bad segment count");
  SegTable tab;
  memset(&tab, 0, sizeof(tab));
  tab.nseg = nseg;
  int64_t row = 0, lone_tiles = 0;
  for (int s = 0; s < nseg; ++s) {
    tab.g[s] = g[s];
    tab.row0[s] = (int)row;
    int rc = seg_map(&tab.tm[s][0], q, row, q_ss, (int64_t)Hq * HD, g[s].S, QT);
    if (!rc) rc = seg_map(&tab.tm[s][1], k, row, k_ss, (int64_t)Hkv * HD, g[s].S, TK);
    if (!rc) rc = seg_map(&tab.tm[s][2], v, row, v_ss, (int64_t)Hkv * HD, g[s].S, TK);
    if (!rc) rc = seg_map(&tab.tm[s][3], dout, row, do_ss, (int64_t)Hq * HD, g[s].S, QT);
    if (rc) return rc;
    row += g[s].S;
    lone_tiles = seg_tiles(g[s]);
  }
  // a unit is a key tile (items: unit x query head, heads fastest); its cost the
  // 64-query steps that read it
  auto cost = [](const PartGeom& sg, int kt) { return query_tiles(sg, kt * TK, QT).count(); };
  int rc = seg_table_order(tab, [](const PartGeom& sg) { return seg_tiles(sg); }, cost);
  if (rc) return rc;
  // light units (at most kGroupSteps steps over all rep heads of a group) run one
  // item per KV head after every per-head unit; stable, so both parts keep the
  // segment-major, heaviest-first order
  const int rep = Hq / Hkv;
  auto light = [&](int s, int kt) { return rep > 1 && cost(tab.g[s], kt) * rep <= kGroupSteps; };
  int64_t units;
  if (tab.nwork > 0) {
    units = tab.nwork;
    auto heavy_w = [&](uint32_t w) {
      return !light((int)(w >> kWorkSegShift), (int)(w & ((1u << kWorkSegShift) - 1)));
    };
    uint32_t* end = std::stable_partition(tab.work, tab.work + tab.nwork, heavy_w);
    tab.nsplit = (int)(end - tab.work);
  } else {
    // a lone segment runs its key tiles in ascending order: the per-head units are
    // the tiles before the first light one
    units = lone_tiles;
    int kt = 0;
    while (kt < lone_tiles && !light(0, kt)) ++kt;
    tab.nsplit = kt;
  }
  PE_CUDA_TRY(cudaFuncSetAttribute(attn_bwd_kv2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)SMEM_KV2));
  const int64_t items = (int64_t)Hq * tab.nsplit + (int64_t)Hkv * (units - tab.nsplit);
  PE_CHECK_ARG(items < (1ll << 31), "attention backward: too many work items");
  const int grid = (int)(items < sm_count() ? items : sm_count());
  attn_bwd_kv2_kernel<<<grid, kThreads, SMEM_KV2, st>>>(tab, lse, delta, dk_acc, dv_acc,
                                                        work_counter, Hq, Hkv, Hq / Hkv,
                                                        1.0f / sqrtf((float)HD), status);
  PE_LAUNCHED();
  return PE_OK;
}

}  // namespace pe
