// Cross-depth masked flash attention backward, dQ half (tcgen05): the backward
// of reference src/pe/nn.py:84-88 under the mask of src/pe/masks.py:43-61,
// partition slot layout (src/pe/partition.py:41-55).
//
// Persistent: one CTA per SM claims units (segment, 128-row query tile, query
// head) from a global counter in work-list order and walks the keys each unit's
// tile reads (the forward's key list) in 64-key steps, query row per TMEM lane:
//   S = Q K^T,  dP = dO V^T                        (N = 64)
//   dS = P (dP - delta),  P = 2^(S c - lse')      (compute warps; bf16 dS
//                                                  packed back over S)
//   dQ += dS K                                     (TMEM accumulator)
// Every MMA takes its A operand from TMEM -- Q and dO are copied there once,
// dS is written there -- so only B (K, V) streams from shared memory, 64 B per
// clock at the full MMA rate; with both operands in shared memory an M = 128
// MMA needs 96-192 B per clock against a shared-memory bandwidth of 128.  The
// 64-key step leaves room to double-buffer S and dP (4 x 64 columns), so the
// MMAs of step j + 1 (and j + 2) run while the compute warps work on step j.
// Across units: the next unit's Q / dO are loaded while the current one runs
// (the shared-memory copy is free once it is in TMEM), and a unit's dQ is scaled
// and stored in bf16 straight from TMEM while the next unit's first S / dP run.
//
// Warp roles (640 threads):
//   warp 0      scheduler + TMA: claims units; Q / dO tile per unit, K / V per
//               step into 4- and 3-deep rings
//   warp 1      tcgen05.mma issue:  dQ(j), S(j+2), dP(j+2) per step
//   warps 2, 3  idle
//   warps 4-19  compute: four per TMEM lane quarter, each owning 16 of the 64
//               key columns (four warps per scheduler hide the TMEM and SFU
//               latency of a step); part p also copies one 64-column half of Q
//               (p = 0, 1) or dO (p = 2, 3) into TMEM and stores 32 of dQ's 128
//               head dims
// TMEM: dQ 0..127, Q 128..191, dO 192..255 (bf16 pairs), S buffers 256 / 320,
//       dP buffers 384 / 448.
#include "attn_tc.cuh"
#include "rope.cuh"

namespace pe {
namespace {

using namespace sm100;
using namespace attn_tc;

constexpr int KT = 64;                         // keys per step
constexpr uint32_t SUB_BYTES = KT * HD * 2;     // 16 KB: 64 rows x 128 bf16
constexpr uint32_t SUB_CHUNK = SUB_BYTES / 2;   // 8 KB: 64 rows x 128 B
constexpr int KS = 4, VS = 3;                  // ring depths
constexpr int kComputeWarps = 16;              // four per TMEM lane quarter
constexpr int kThreads = 128 + 32 * kComputeWarps;
constexpr int kParts = kComputeWarps / 4;
constexpr int kCols = KT / kParts;             // key columns per compute warp

constexpr uint32_t OFF_Q = 0;
constexpr uint32_t OFF_DO = OFF_Q + TILE_BYTES;
constexpr uint32_t OFF_K = OFF_DO + TILE_BYTES;
constexpr uint32_t OFF_V = OFF_K + KS * SUB_BYTES;
constexpr uint32_t OFF_ITEM = OFF_V + VS * SUB_BYTES;  // int [2]
constexpr uint32_t OFF_BAR = OFF_ITEM + 16;
constexpr int NBARS = 2 + 2 + 1 + 1 + 2 * KS + 2 * VS + 2 + 2 + 2 + 1;
constexpr uint32_t OFF_TMEM = OFF_BAR + NBARS * 8;
constexpr size_t SMEM_Q2 = 1024 + OFF_TMEM + 16;

struct Bars {
  uint64_t *item_full, *item_empty, *qdo_full, *qdo_copied, *k_full, *k_empty, *v_full,
      *v_empty, *s_full, *dp_full, *ds_full, *dq_full;
  __device__ explicit Bars(uint64_t* b) {
    item_full = b; b += 2;
    item_empty = b; b += 2;
    qdo_full = b; b += 1;
    qdo_copied = b; b += 1;
    k_full = b; b += KS;
    k_empty = b; b += KS;
    v_full = b; b += VS;
    v_empty = b; b += VS;
    s_full = b; b += 2;
    dp_full = b; b += 2;
    ds_full = b; b += 2;
    dq_full = b; b += 1;
  }
};

// packed dS: the keys of compute part p (columns [p C, p C + C)) sit in columns
// [p C, p C + C / 2) of their S buffer, which only part p writes
__device__ __forceinline__ uint32_t a_col(int kk) {
  constexpr int steps = kCols / 16;
  return (uint32_t)((kk / steps) * kCols + (kk % steps) * 8);
}

// a work unit (segment, 128-row query tile, query head) and the 64-key steps it walks
struct Unit {
  int seg, h, q0, r_end, m_beg, m_end, n;
  PartGeom g;
  int64_t r0;  // first stacked row of the segment
  __device__ Unit(int w, int Hq, const SegTable& tab) {
    const int e = w / Hq;
    h = w - e * Hq;
    int qt;
    if (tab.nwork > 0) {
      unpack_work(tab.work[e], seg, qt);
    } else {  // a lone segment: its last (heaviest) tile first
      seg = 0;
      qt = (tab.g[0].S + TQ - 1) / TQ - 1 - e;
    }
    g = tab.g[seg];
    r0 = tab.row0[seg];
    q0 = qt * TQ;
    key_tiles(g, q0, r_end, m_beg, m_end, KT);
    n = r_end + (m_end - m_beg);
  }
  __device__ __forceinline__ int key(int j) const {
    return (j < r_end ? j : m_beg + (j - r_end)) * KT;
  }
};

__global__ void __launch_bounds__(kThreads, 1)
attn_bwd_q2_kernel(const __grid_constant__ SegTable tab, const float* __restrict__ lse,
                   const float* __restrict__ delta, __nv_bfloat16* __restrict__ dq, int64_t dq_ss,
                   const __nv_bfloat16* __restrict__ rope_cs, int64_t cs_ld, int Hq, int rep,
                   float scale, int total, int* work_counter, int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  Bars B(reinterpret_cast<uint64_t*>(smem + OFF_BAR));
  volatile int* sItem = reinterpret_cast<volatile int*>(smem + OFF_ITEM);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_TMEM);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&B.item_full[i], 1);
      mbar_init(&B.item_empty[i], 1 + kComputeWarps);  // MMA warp, compute warps
    }
    mbar_init(B.qdo_full, 1);
    mbar_init(B.qdo_copied, kComputeWarps);
    for (int i = 0; i < KS; ++i) {
      mbar_init(&B.k_full[i], 1);
      mbar_init(&B.k_empty[i], 1);
    }
    for (int i = 0; i < VS; ++i) {
      mbar_init(&B.v_full[i], 1);
      mbar_init(&B.v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&B.s_full[i], 1);
      mbar_init(&B.dp_full[i], 1);
      // scores run up to two steps ahead, so a fast warp may reach step j + 1
      // before a slow one arrives for step j (never step j + 2)
      mbar_init(&B.ds_full[i], kComputeWarps);
    }
    mbar_init(B.dq_full, 1);
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
  const uint32_t tDQ = tmem, tQ = tmem + 128, tDO = tmem + 192, tS = tmem + 256,
                 tDP = tmem + 384;

  // every role walks the same unit sequence; `ic` counts units, `gs` steps
  auto read_item = [&](int ic, bool& ok) -> int {
    if (!mbar_wait(&B.item_full[ic & 1], (ic >> 1) & 1, status, 371)) {
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
        if (!mbar_wait(&B.item_empty[ic & 1], ((ic >> 1) & 1) ^ 1u, status, 372)) { ok = false; break; }
        sItem[ic & 1] = w;
        mbar_arrive(&B.item_full[ic & 1]);  // release: publishes the slot write
        if (w < 0) break;
        const Unit u(w, Hq, tab);
        const CUtensorMap* tmQ = &tab.tm[u.seg][0];
        const CUtensorMap* tmK = &tab.tm[u.seg][1];
        const CUtensorMap* tmV = &tab.tm[u.seg][2];
        const CUtensorMap* tmDO = &tab.tm[u.seg][3];
        const int kvh = u.h / rep;
        // Q / dO once the compute warps copied the previous unit's into TMEM
        if (!mbar_wait(B.qdo_copied, (ic & 1) ^ 1u, status, 373)) { ok = false; break; }
        mbar_arrive_expect_tx(B.qdo_full, 2 * TILE_BYTES);
        tma_load_2d(smem + OFF_Q, tmQ, B.qdo_full, u.h * HD, u.q0);
        tma_load_2d(smem + OFF_Q + CHUNK, tmQ, B.qdo_full, u.h * HD + 64, u.q0);
        tma_load_2d(smem + OFF_DO, tmDO, B.qdo_full, u.h * HD, u.q0);
        tma_load_2d(smem + OFF_DO + CHUNK, tmDO, B.qdo_full, u.h * HD + 64, u.q0);
        last_bar = B.qdo_full;
        last_ph = ic & 1;
        for (int j = 0; j < u.n && ok; ++j) {
          const int gj = gs + j, k0 = u.key(j);
          const int ks = gj % KS, vs = gj % VS;
          if (!mbar_wait(&B.k_empty[ks], ((gj / KS) & 1) ^ 1u, status, 360)) { ok = false; break; }
          uint8_t* kd = smem + OFF_K + ks * SUB_BYTES;
          mbar_arrive_expect_tx(&B.k_full[ks], SUB_BYTES);
          tma_load_2d(kd, tmK, &B.k_full[ks], kvh * HD, k0);
          tma_load_2d(kd + SUB_CHUNK, tmK, &B.k_full[ks], kvh * HD + 64, k0);
          last_bar = &B.k_full[ks];
          last_ph = (gj / KS) & 1;
          if (!mbar_wait(&B.v_empty[vs], ((gj / VS) & 1) ^ 1u, status, 361)) { ok = false; break; }
          uint8_t* vd = smem + OFF_V + vs * SUB_BYTES;
          mbar_arrive_expect_tx(&B.v_full[vs], SUB_BYTES);
          tma_load_2d(vd, tmV, &B.v_full[vs], kvh * HD, k0);
          tma_load_2d(vd + SUB_CHUNK, tmV, &B.v_full[vs], kvh * HD + 64, k0);
          last_bar = &B.v_full[vs];
          last_ph = (gj / VS) & 1;
        }
        if (!ok) break;
        gs += u.n;
      }
      // on a failed wait, let this thread's last copy land before the CTA exits
      if (!ok && last_bar) mbar_wait(last_bar, last_ph, nullptr, 0);
    }
  } else if (warp == 1) {
    // ---------------- MMA issue ----------------
    constexpr uint32_t ID_SP = idesc_bf16(TQ, KT, false, false);  // S, dP (A = Q / dO)
    constexpr uint32_t ID_DQ = idesc_bf16(TQ, HD, false, true);   // dQ += dS K
    bool ok = true;
    int gs = 0;
    for (int ic = 0; ok; ++ic) {
      const int w = read_item(ic, ok);
      if (w < 0) break;
      const bool leader = elect_one();
      const int leader_lane = __ffs(__ballot_sync(0xffffffffu, leader)) - 1;
      if (leader) {
        const Unit u(w, Hq, tab);
        // S(gj) = Q K(gj)^T and dP(gj) = dO V(gj)^T into buffers gj & 1
        auto issue_scores = [&](int gj) -> bool {
          const int ks = gj % KS, vs = gj % VS, b = gj & 1;
          if (!mbar_wait(&B.k_full[ks], (gj / KS) & 1, status, 363)) return false;
          tc_fence_after();
          const uint32_t k_base = smem_u32(smem + OFF_K + ks * SUB_BYTES);
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk)
            mma_bf16_ts(tS + b * KT, tQ + kk * 8,
                        sw128_desc(k_base + (kk >> 2) * SUB_CHUNK + (kk & 3) * 32, 16, 1024),
                        ID_SP, kk > 0 ? 1u : 0u);
          mma_commit(&B.s_full[b]);
          if (!mbar_wait(&B.v_full[vs], (gj / VS) & 1, status, 364)) return false;
          tc_fence_after();
          const uint32_t v_base = smem_u32(smem + OFF_V + vs * SUB_BYTES);
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk)
            mma_bf16_ts(tDP + b * KT, tDO + kk * 8,
                        sw128_desc(v_base + (kk >> 2) * SUB_CHUNK + (kk & 3) * 32, 16, 1024),
                        ID_SP, kk > 0 ? 1u : 0u);
          mma_commit(&B.dp_full[b]);
          mma_commit(&B.v_empty[vs]);  // V(gj) has no other reader
          return true;
        };
        // this unit's Q / dO in TMEM (the S / dP buffers it overwrites were read by
        // the previous unit's dQ MMAs, issued before)
        ok = mbar_wait(B.qdo_copied, ic & 1, status, 365);
        if (ok) {
          tc_fence_after();
          for (int j = 0; j < 2 && j < u.n && ok; ++j) ok = issue_scores(gs + j);
        }
        for (int j = 0; j < u.n && ok; ++j) {
          const int gj = gs + j, b = gj & 1, ks = gj % KS;
          // dS(gj) from every compute warp; each drained the previous unit's dQ first,
          // so the unit's first dQ MMA (which overwrites the accumulator) may go
          if (!mbar_wait(&B.ds_full[b], (gj >> 1) & 1, status, 366)) { ok = false; break; }
          tc_fence_after();
          const uint32_t k_base = smem_u32(smem + OFF_K + ks * SUB_BYTES);
#pragma unroll
          for (int kk = 0; kk < KT / 16; ++kk)
            mma_bf16_ts(tDQ, tS + b * KT + a_col(kk),
                        sw128_desc(k_base + kk * 2048, SUB_CHUNK, 1024), ID_DQ,
                        (j > 0 || kk > 0) ? 1u : 0u);
          mma_commit(&B.k_empty[ks]);
          // S(j+2) / dP(j+2) overwrite buffer b after dQ(j) read dS(j) (in order)
          if (j + 2 < u.n && !issue_scores(gj + 2)) { ok = false; break; }
        }
        if (ok) mma_commit(B.dq_full);
        gs += u.n;
      }
      __syncwarp();
      ok = __shfl_sync(0xffffffffu, ok, leader_lane);
      gs = __shfl_sync(0xffffffffu, gs, leader_lane);
    }
  } else if (warp >= 4) {
    // ---------------- compute: thread = query row (TMEM lane) ----------------
    constexpr int C = kCols;
    const int quarter = warp & 3;
    const int part = (warp - 4) >> 2;
    const int cb = part * C;
    const int row = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const float scale_log2 = scale * kLog2e;
    const float2 sc2 = make_float2(scale_log2, scale_log2);
    bool ok = true;
    int gs = 0;
    // the previous unit's dQ row, written once that unit's last dQ MMA completed:
    // this part's head dims [16 part, 16 part + 16) and their rotary partners 64 on,
    // rounded to bf16 and, with a cos / sin table, rotated back by the transpose of
    // the rotary embedding (the gradient with respect to the unrotated q)
    __nv_bfloat16* pending = nullptr;
    const __nv_bfloat16* pending_cs = nullptr;
    bool have_pending = false;
    auto drain = [&](int ic_prev) -> bool {
      if (!mbar_wait(B.dq_full, ic_prev & 1, status, 370)) return false;
      tc_fence_after();
      float va[16], vb[16];
      tmem_ld16(tDQ + lane_off + part * 16, va);
      tmem_ld16(tDQ + lane_off + 64 + part * 16, vb);
      tmem_wait_ld();
      if (pending) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          va[i] = rb16(va[i] * scale);
          vb[i] = rb16(vb[i] * scale);
        }
        if (pending_cs) {
          float c[16], sn[16];
          load_bf16_f32<16>(pending_cs + part * 16, c);
          load_bf16_f32<16>(pending_cs + 64 + part * 16, sn);
#pragma unroll
          for (int i = 0; i < 16; ++i) rope_rotate_pair(va[i], vb[i], c[i], sn[i], true);
        }
        // each half's 32 bytes as two back-to-back stores: whole sectors after L1 merging
        uint4* da = reinterpret_cast<uint4*>(pending + part * 16);
#pragma unroll
        for (int q = 0; q < 2; ++q)
          da[q] = make_uint4(pack_bf16x2(va[8 * q], va[8 * q + 1]), pack_bf16x2(va[8 * q + 2], va[8 * q + 3]),
                             pack_bf16x2(va[8 * q + 4], va[8 * q + 5]), pack_bf16x2(va[8 * q + 6], va[8 * q + 7]));
        uint4* db = reinterpret_cast<uint4*>(pending + 64 + part * 16);
#pragma unroll
        for (int q = 0; q < 2; ++q)
          db[q] = make_uint4(pack_bf16x2(vb[8 * q], vb[8 * q + 1]), pack_bf16x2(vb[8 * q + 2], vb[8 * q + 3]),
                             pack_bf16x2(vb[8 * q + 4], vb[8 * q + 5]), pack_bf16x2(vb[8 * q + 6], vb[8 * q + 7]));
      }
      return true;
    };
    int ic = 0;
    for (; ok; ++ic) {
      const int w = read_item(ic, ok);
      if (w < 0) break;
      const Unit u(w, Hq, tab);
      // ---- this unit's Q (parts 0, 1) or dO (parts 2, 3) half row -> TMEM as bf16
      // pairs (A operand).  The previous unit's S / dP MMAs, which read the old
      // copy, have all completed: this warp waited for its last dP. ----
      if (!mbar_wait(B.qdo_full, ic & 1, status, 367)) { ok = false; break; }
      {
        const int ch = part & 1;
        const uint8_t* src = smem + (part < 2 ? OFF_Q : OFF_DO) + ch * CHUNK;
        uint32_t r32[32];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const uint4 x = *reinterpret_cast<const uint4*>(src + swz(row, q));
          r32[q * 4 + 0] = x.x;
          r32[q * 4 + 1] = x.y;
          r32[q * 4 + 2] = x.z;
          r32[q * 4 + 3] = x.w;
        }
        tmem_st32((part < 2 ? tQ : tDO) + lane_off + ch * 32, r32);
        tmem_wait_st();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(B.qdo_copied);
      // ---- the previous unit's dQ, while this unit's first S / dP run ----
      if (have_pending && !drain(ic - 1)) { ok = false; break; }
      const int s = u.q0 + row;
      const bool valid = s < u.g.S;
      int qi = -1, qd = 0;
      float l2 = 0.f, dl = 0.f;
      if (valid) {
        const int64_t li = (int64_t)Hq * u.r0 + (int64_t)u.h * u.g.S + s;
        decode(u.g, s, qi, qd);
        l2 = lse[li] * kLog2e;
        dl = delta[li];
      }
      const int lo = qd > 0 ? u.g.a1 + (qi - u.g.a0) * u.g.km1 : 0;
      const float2 nl2 = make_float2(-l2, -l2), ndl2 = make_float2(-dl, -dl);
      pending = valid ? dq + (u.r0 + s) * dq_ss + u.h * HD : nullptr;
      pending_cs = valid && rope_cs ? rope_cs + (u.r0 + s) * cs_ld : nullptr;
      have_pending = true;
      for (int j = 0; j < u.n; ++j) {
        const int gj = gs + j, b = gj & 1;
        const int k0 = u.key(j) + cb;
        if (!mbar_wait(&B.s_full[b], (gj >> 1) & 1, status, 368)) { ok = false; break; }
        tc_fence_after();
        float sv[C];
        tmem_ld16(tS + b * KT + lane_off + cb, sv);
        tmem_wait_ld();
        // P = 2^(S c - lse') (masked pairs exactly 0)
        if (k0 + C - 1 <= qi) {  // every key of this warp's slice is real and <= the anchor
#pragma unroll
          for (int c = 0; c < C; c += 2) {
            const float2 a = fma2(make_float2(sv[c], sv[c + 1]), sc2, nl2);
            sv[c] = ex2_approx(a.x);
            sv[c + 1] = ex2_approx(a.y);
          }
        } else {
#pragma unroll
          for (int c = 0; c < C; ++c) {
            const int ks = k0 + c;
            const bool allow = ks <= qi || (unsigned)(ks - lo) < (unsigned)qd;
            sv[c] = allow ? ex2_approx(fmaf(sv[c], scale_log2, -l2)) : 0.f;
          }
        }
        if (!mbar_wait(&B.dp_full[b], (gj >> 1) & 1, status, 369)) { ok = false; break; }
        tc_fence_after();
        float dv[C];
        tmem_ld16(tDP + b * KT + lane_off + cb, dv);
        tmem_wait_ld();
        uint32_t pw[C / 2];
#pragma unroll
        for (int c = 0; c < C; c += 2) {
          const float2 a =
              mul2(make_float2(sv[c], sv[c + 1]), add2(make_float2(dv[c], dv[c + 1]), ndl2));
          pw[c / 2] = pack_bf16x2(a.x, a.y);
        }
        tmem_st8(tS + b * KT + lane_off + cb, pw);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&B.ds_full[b]);
      }
      if (!ok) break;
      gs += u.n;
    }
    // the last unit's dQ
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

int attn_bwd_q2_launch(int nseg, const PartGeom* g, int Hq, int Hkv, const void* q,
                       int64_t q_ss, const void* k, int64_t k_ss, const void* v, int64_t v_ss,
                       const void* dout, int64_t do_ss, const float* lse, const float* delta,
                       void* dq, int64_t dq_ss, const void* rope_cs, int64_t cs_ld,
                       int* work_counter, int* status, cudaStream_t st) {
  PE_CHECK_ARG(nseg >= 1 && nseg <= kMaxSeg, "attention backward: bad segment count");
  SegTable tab;
  memset(&tab, 0, sizeof(tab));
  tab.nseg = nseg;
  int64_t row = 0;
  int max_units = 0;
  for (int s = 0; s < nseg; ++s) {
    tab.g[s] = g[s];
    tab.row0[s] = (int)row;
    int rc = seg_map(&tab.tm[s][0], q, row, q_ss, (int64_t)Hq * HD, g[s].S, TQ);
    if (!rc) rc = seg_map(&tab.tm[s][1], k, row, k_ss, (int64_t)Hkv * HD, g[s].S, KT);
    if (!rc) rc = seg_map(&tab.tm[s][2], v, row, v_ss, (int64_t)Hkv * HD, g[s].S, KT);
    if (!rc) rc = seg_map(&tab.tm[s][3], dout, row, do_ss, (int64_t)Hq * HD, g[s].S, TQ);
    if (rc) return rc;
    row += g[s].S;
    max_units = std::max(max_units, seg_tiles(g[s]));
  }
  // a unit is a query tile; its cost the 64-key steps it walks
  auto cost = [](const PartGeom& sg, int qt) {
    int r_end, m_beg, m_end;
    key_tiles(sg, qt * TQ, r_end, m_beg, m_end, KT);
    return r_end + (m_end - m_beg);
  };
  int rc = seg_table_order(tab, [](const PartGeom& sg) { return seg_tiles(sg); }, cost);
  if (rc) return rc;
  // units: (work-list entry or, for a lone segment, query tile) x query head,
  // claimed from *work_counter by one persistent CTA per SM
  const int64_t units = (int64_t)Hq * (tab.nwork > 0 ? tab.nwork : max_units);
  PE_CHECK_ARG(units < (1ll << 31), "attention backward: too many query tiles");
  PE_CUDA_TRY(cudaFuncSetAttribute(attn_bwd_q2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)SMEM_Q2));
  const int grid = (int)(units < sm_count() ? units : sm_count());
  attn_bwd_q2_kernel<<<grid, kThreads, SMEM_Q2, st>>>(tab, lse, delta, (__nv_bfloat16*)dq, dq_ss,
                                                      (const __nv_bfloat16*)rope_cs, cs_ld, Hq,
                                                      Hq / Hkv, 1.0f / sqrtf((float)HD),
                                                      (int)units, work_counter, status);
  PE_LAUNCHED();
  return PE_OK;
}

}  // namespace pe
