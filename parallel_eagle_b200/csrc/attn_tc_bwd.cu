// Cross-depth masked flash attention on the 5th-generation tensor cores
// (backward): dQ, dK, dV for bf16, head_dim 128, partition slot layout
// (the backward of reference src/pe/nn.py:84-88 under the mask of
// src/pe/masks.py:43-61).
//
// One CTA = one 128-slot key tile x one query head.  It loops over the query
// tiles whose rows can see any key of the tile (the rule's key-side view: a real
// key j is read by the real rows j.. and every prediction row of anchors >= j;
// a prediction key (i, e) only by the rows (i, d >= e)).  Per query tile, with
// the key on TMEM lanes:
//   S^T  = K Q^T          dP^T = V dO^T               (tcgen05, TMEM)
//   P^T  = exp(scale S^T - lse)   dS^T = P^T (dP^T - delta)   (softmax warps,
//          bf16 to shared memory; masked pairs are exactly zero; tiles the rule
//          fully allows skip the per-pair test)
//   dV  += P^T dO         dK  += dS^T Q               (TMEM accumulators)
//   dQ_part = dS K        -> fp32 vector atomics into a dQ accumulator
// At the end the head's dK/dV tile is added (fp32 atomics) into the KV head's
// accumulator, so the 7 query heads of a GQA group reduce without any K/V
// expansion; a final pass scales and casts dQ, dK, dV to bf16.
//
// TMEM columns: dK 0..127, dV 128..255, S^T (then dQ_part) 256..383, dP^T 384..511.
#include "attn_tc.cuh"
#include "rope.cuh"

namespace pe {
namespace {

using namespace sm100;
using namespace attn_tc;

// warp 0 TMA, warp 1 MMA, warps 2..9 softmax/epilogue: two warps per TMEM lane
// quarter, each owning 64 of the 128 query (or head-dim) columns
constexpr int kThreads = 320;
constexpr int kSoftmaxThreads = 256;
// K, V, Q, dO, P^T, dS^T tiles + per-query (lse, delta, anchor, depth) x 2 buffers
constexpr size_t SMEM_BWD = 1024 + 6 * TILE_BYTES + 2 * 4 * TQ * 4 + 256;

__device__ __forceinline__ void named_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__global__ void __launch_bounds__(kThreads, 1)
attn_bwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                   const float* __restrict__ lse, const float* __restrict__ delta,
                   float* __restrict__ dq_acc, float* __restrict__ dk_acc,
                   float* __restrict__ dv_acc, PartGeom g, int Hq, int Hkv, int rep, float scale,
                   int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sK = smem;
  uint8_t* sV = sK + TILE_BYTES;
  uint8_t* sQ = sV + TILE_BYTES;
  uint8_t* sDO = sQ + TILE_BYTES;
  uint8_t* sP = sDO + TILE_BYTES;   // P^T  [key rows][query cols]
  uint8_t* sDS = sP + TILE_BYTES;   // dS^T [key rows][query cols]
  float* sL = reinterpret_cast<float*>(sDS + TILE_BYTES);  // [2][TQ] lse * log2(e)
  float* sD = sL + 2 * TQ;                                  // [2][TQ] delta
  int* sA = reinterpret_cast<int*>(sD + 2 * TQ);            // [2][TQ] query anchor
  int* sDp = sA + 2 * TQ;                                   // [2][TQ] query depth
  uint64_t* bars = reinterpret_cast<uint64_t*>(sDp + 2 * TQ);
  uint64_t* kv_full = bars + 0;
  uint64_t* qdo_full = bars + 1;
  uint64_t* qdo_empty = bars + 2;
  uint64_t* s_full = bars + 3;
  uint64_t* p_full = bars + 4;
  uint64_t* mm_done = bars + 5;
  uint64_t* dq_read = bars + 6;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 7);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // grid (head, key tile): low key tiles are read by the most query tiles, and blocks
  // dispatch head-fastest, so the heaviest tiles of every head start first
  const int kt = blockIdx.y;
  const int h = blockIdx.x;
  const int kvh = h / rep;
  const int k0 = kt * TK;
  const Ranges qr = query_tiles(g, k0);
  const int n_it = qr.count();

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    mbar_init(qdo_full, 1);
    mbar_init(qdo_empty, 1);
    mbar_init(s_full, 1);
    mbar_init(p_full, 8);
    mbar_init(mm_done, 1);
    mbar_init(dq_read, 8);
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
  const uint32_t tDK = tmem, tDV = tmem + 128, tS = tmem + 256, tDP = tmem + 384;

  if (warp == 0) {
    if (elect_one()) {
      bool ok = true;
      int issued = 0;
      mbar_arrive_expect_tx(kv_full, 2 * TILE_BYTES);
      tma_load_2d(sK, &tmK, kv_full, kvh * HD, k0);
      tma_load_2d(sK + CHUNK, &tmK, kv_full, kvh * HD + 64, k0);
      tma_load_2d(sV, &tmV, kv_full, kvh * HD, k0);
      tma_load_2d(sV + CHUNK, &tmV, kv_full, kvh * HD + 64, k0);
      for (int it = 0; it < n_it && ok; ++it) {
        if (!mbar_wait(qdo_empty, (it & 1) ^ 1u, status, 301)) { ok = false; break; }
        const int q0 = qr.at(it) * TQ;
        mbar_arrive_expect_tx(qdo_full, 2 * TILE_BYTES);
        tma_load_2d(sQ, &tmQ, qdo_full, h * HD, q0);
        tma_load_2d(sQ + CHUNK, &tmQ, qdo_full, h * HD + 64, q0);
        tma_load_2d(sDO, &tmDO, qdo_full, h * HD, q0);
        tma_load_2d(sDO + CHUNK, &tmDO, qdo_full, h * HD + 64, q0);
        issued = it + 1;
      }
      mbar_wait(kv_full, 0, nullptr, 0);
      if (issued > 0) mbar_wait(qdo_full, (issued - 1) & 1, nullptr, 0);
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t ID_KK = idesc_bf16(TK, TQ, false, false);  // S^T, dP^T
      constexpr uint32_t ID_KM = idesc_bf16(TK, HD, false, true);   // dV, dK
      constexpr uint32_t ID_MM = idesc_bf16(TQ, HD, true, true);    // dQ
      const uint32_t k_base = smem_u32(sK), v_base = smem_u32(sV), q_base = smem_u32(sQ);
      const uint32_t do_base = smem_u32(sDO), p_base = smem_u32(sP), ds_base = smem_u32(sDS);
      bool ok = mbar_wait(kv_full, 0, status, 302);
      for (int it = 0; it < n_it && ok; ++it) {
        if (!mbar_wait(qdo_full, it & 1, status, 303)) { ok = false; break; }
        if (it > 0 && !mbar_wait(dq_read, (it - 1) & 1, status, 304)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * CHUNK + (kk & 3) * 32;
          mma_bf16_ss(tS, sw128_desc(k_base + off, 16, 1024), sw128_desc(q_base + off, 16, 1024),
                      ID_KK, kk > 0 ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * CHUNK + (kk & 3) * 32;
          mma_bf16_ss(tDP, sw128_desc(v_base + off, 16, 1024), sw128_desc(do_base + off, 16, 1024),
                      ID_KK, kk > 0 ? 1u : 0u);
        }
        mma_commit(s_full);
        if (!mbar_wait(p_full, it & 1, status, 305)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < TQ / 16; ++kk) {
          const uint32_t aoff = (kk >> 2) * CHUNK + (kk & 3) * 32;  // K-major over queries
          const uint32_t boff = kk * 2048;                          // MN-major, 16 rows per step
          const uint32_t acc = (it > 0 || kk > 0) ? 1u : 0u;
          mma_bf16_ss(tDV, sw128_desc(p_base + aoff, 16, 1024),
                      sw128_desc(do_base + boff, CHUNK, 1024), ID_KM, acc);
          mma_bf16_ss(tDK, sw128_desc(ds_base + aoff, 16, 1024),
                      sw128_desc(q_base + boff, CHUNK, 1024), ID_KM, acc);
        }
#pragma unroll
        for (int kk = 0; kk < TK / 16; ++kk) {
          const uint32_t off = kk * 2048;  // both MN-major, 16 key rows per step
          mma_bf16_ss(tS, sw128_desc(ds_base + off, CHUNK, 1024),
                      sw128_desc(k_base + off, CHUNK, 1024), ID_MM, kk > 0 ? 1u : 0u);
        }
        mma_commit(qdo_empty);
        mma_commit(mm_done);
      }
    }
  } else {
    // ---------------- softmax / epilogue warps (256 threads) ----------------
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;  // warps 2..5 -> 0, 6..9 -> 1
    const int cb = half * 64;          // query columns (softmax) / head-dim columns (epilogues)
    const int row = quarter * 32 + lane;  // TMEM lane: key row (S^T, dP^T, dK, dV) / query row (dQ)
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const int kj = k0 + row;
    const bool kvalid = kj < g.S;
    int ka = 0, ke = 0;
    if (kvalid) decode(g, kj, ka, ke);
    const float scale_log2 = scale * kLog2e;
    const int64_t dq_ld = (int64_t)Hq * HD;
    bool ok = true;
    for (int it = 0; it < n_it; ++it) {
      const int q0 = qr.at(it) * TQ;
      const int buf = it & 1;
      const bool full = tile_fully_allowed(g, q0, k0);
      if (half == 0) {
        // per-query operands of this tile, one per thread of the first half
        const int q = q0 + row;
        float lv = INFINITY, dl = 0.f;
        int qa = -1, qd = 0;
        if (q < g.S) {
          lv = lse[(int64_t)h * g.S + q] * kLog2e;
          dl = delta[(int64_t)h * g.S + q];
          decode(g, q, qa, qd);
        }
        sL[buf * TQ + row] = lv;
        sD[buf * TQ + row] = dl;
        sA[buf * TQ + row] = qa;
        sDp[buf * TQ + row] = qd;
      }
      named_sync(1, kSoftmaxThreads);
      if (!mbar_wait(s_full, it & 1, status, 306)) { ok = false; break; }
      tc_fence_after();
      const float* L2 = sL + buf * TQ;
      const float* DL = sD + buf * TQ;
      const int* QA = sA + buf * TQ;
      const int* QD = sDp + buf * TQ;
#pragma unroll 1
      for (int c0 = cb; c0 < cb + 64; c0 += 32) {
        float sv[32], dpv[32];
        tmem_ld32(tS + lane_off + c0, sv);
        tmem_ld32(tDP + lane_off + c0, dpv);
        tmem_wait_ld();
        uint32_t pw[16], dw[16];
        if (full) {
#pragma unroll
          for (int c = 0; c < 32; c += 2) {
            const float p0 = exp2f(sv[c] * scale_log2 - L2[c0 + c]);
            const float p1 = exp2f(sv[c + 1] * scale_log2 - L2[c0 + c + 1]);
            pw[c / 2] = pack_bf16x2(p0, p1);
            dw[c / 2] = pack_bf16x2(p0 * (dpv[c] - DL[c0 + c]), p1 * (dpv[c + 1] - DL[c0 + c + 1]));
          }
        } else {
#pragma unroll
          for (int c = 0; c < 32; c += 2) {
            float pp[2], dd[2];
#pragma unroll
            for (int t = 0; t < 2; ++t) {
              const int qc = c0 + c + t;
              const int qa = QA[qc];
              const bool allow = kvalid && qa >= 0 &&
                                 (ke == 0 ? (ka <= qa) : (ka == qa && ke <= QD[qc]));
              const float p = allow ? exp2f(sv[c + t] * scale_log2 - L2[qc]) : 0.f;
              pp[t] = p;
              dd[t] = p * (dpv[c + t] - DL[qc]);
            }
            pw[c / 2] = pack_bf16x2(pp[0], pp[1]);
            dw[c / 2] = pack_bf16x2(dd[0], dd[1]);
          }
        }
        const int ch = c0 >> 6;
        const int u0 = (c0 & 63) >> 3;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const uint32_t off = ch * CHUNK + swz(row, u0 + u);
          *reinterpret_cast<uint4*>(sP + off) =
              make_uint4(pw[4 * u], pw[4 * u + 1], pw[4 * u + 2], pw[4 * u + 3]);
          *reinterpret_cast<uint4*>(sDS + off) =
              make_uint4(dw[4 * u], dw[4 * u + 1], dw[4 * u + 2], dw[4 * u + 3]);
        }
      }
      fence_proxy_async();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
      // dQ partial (query row per TMEM lane) -> fp32 atomics
      if (!mbar_wait(mm_done, it & 1, status, 307)) { ok = false; break; }
      tc_fence_after();
      const int q = q0 + row;
#pragma unroll 1
      for (int c0 = cb; c0 < cb + 64; c0 += 32) {
        float v[32];
        tmem_ld32(tS + lane_off + c0, v);
        tmem_wait_ld();
        if (q < g.S) atomic_add_row32(dq_acc + (int64_t)q * dq_ld + h * HD + c0, v, 1.f);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(dq_read);
    }
    // this head's dK, dV tile (key row per TMEM lane) -> the KV head's fp32 accumulators
    if (ok && n_it > 0) {
      const int64_t kv_ld = (int64_t)Hkv * HD;
#pragma unroll 1
      for (int c0 = cb; c0 < cb + 64; c0 += 32) {
        float v[32];
        tmem_ld32(tDK + lane_off + c0, v);
        tmem_wait_ld();
        if (kvalid) atomic_add_row32(dk_acc + (int64_t)kj * kv_ld + kvh * HD + c0, v, 1.f);
        tmem_ld32(tDV + lane_off + c0, v);
        tmem_wait_ld();
        if (kvalid) atomic_add_row32(dv_acc + (int64_t)kj * kv_ld + kvh * HD + c0, v, 1.f);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------------ //
// Split backward (no dQ atomics):
//
// attn_bwd_q_kernel: one CTA = one 128-row query tile of one head, walking the
// key tiles the tile reads (the forward's list).  Per key tile:
//   S = Q K^T, dP = dO V^T (TMEM);  P = 2^(S c - lse'), dS = P (dP - delta) in
//   registers (query row per TMEM lane); dS (bf16) written back over S and read
//   by the A-from-TMEM MMA  dQ += dS K;  dQ stays in TMEM for the whole tile and
//   is stored once, scaled, in bf16.  S is double-buffered, so S(j+1) runs while
//   the softmax warps work on tile j.
//   TMEM: dQ 0..127, dP 128..255, S 256..383 / 384..511.
//
// attn_bwd_kv_kernel: one CTA = one 128-key tile of one query head, walking the
// query tiles that read it.  Per query tile:
//   S^T = K Q^T, dP^T = V dO^T (TMEM); P^T written back over S^T, then
//   dS^T = P^T (dP^T - delta) over dP^T; dV += P^T dO starts as soon as P^T is
//   in place and overlaps the dS^T arithmetic, then dK += dS^T Q.  The head's
//   dK / dV tile is added (fp32) into the KV head's accumulator at the end.
//   TMEM: dK 0..127, dV 128..255, S^T 256..383, dP^T 384..511.
// ------------------------------------------------------------------------ //
// dK/dV kernel: four compute warps per TMEM lane quarter, each owning 32 of the
// 128 query columns (more warps in flight to hide TMEM and SFU latency)
constexpr int kKvParts = 4;
constexpr int kKvThreads = 64 + 128 * kKvParts;
constexpr int kKvCols = TQ / kKvParts;
constexpr size_t SMEM_BWD_Q = 1024 + 2 * TILE_BYTES /*Q, dO*/ + 2 * 2 * TILE_BYTES /*K,V x2*/ + 256;
constexpr size_t SMEM_BWD_KV = 1024 + 2 * TILE_BYTES /*K, V*/ + 2 * 2 * TILE_BYTES /*Q,dO x2*/ +
                               2 * 4 * TQ * 4 /*per-query operands x2*/ + 256;

__global__ void __launch_bounds__(kKvThreads, 1)
attn_bwd_q_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                  const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                  const float* __restrict__ lse, const float* __restrict__ delta,
                  __nv_bfloat16* __restrict__ dq, int64_t dq_ss, PartGeom g, int rep, float scale,
                  int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sDO = sQ + TILE_BYTES;
  uint8_t* sKV = sDO + TILE_BYTES;  // stage s: K at + s * 2 * TILE, V at + TILE
  uint64_t* bars = reinterpret_cast<uint64_t*>(sKV + 4 * TILE_BYTES);
  uint64_t* qdo_full = bars + 0;
  uint64_t* kv_full = bars + 1;   // [2]
  uint64_t* kv_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;    // [2] S(j) and dP(j) computed
  uint64_t* dp_free = bars + 7;   // dP(j) read by the softmax warps
  uint64_t* ds_full = bars + 8;   // dS(j) written over S(j)
  uint64_t* dq_full = bars + 9;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 10);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_qt = (g.S + TQ - 1) / TQ;
  // grid (head, tile): blocks dispatch head-fastest, so the heaviest tiles of every
  // head start first
  const int qt = num_qt - 1 - (int)blockIdx.y;
  const int h = blockIdx.x;
  const int kvh = h / rep;
  const int q0 = qt * TQ;
  int r_end, m_beg, m_end;
  key_tiles(g, q0, r_end, m_beg, m_end);
  const int n = r_end + (m_end - m_beg);
  auto tile_at = [&](int j) { return j < r_end ? j : m_beg + (j - r_end); };

  if (threadIdx.x == 0) {
    mbar_init(qdo_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
    }
    mbar_init(dp_free, 4 * kKvParts);
    mbar_init(ds_full, 4 * kKvParts);
    mbar_init(dq_full, 1);
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
  const uint32_t tDQ = tmem, tDP = tmem + 128, tS = tmem + 256;

  if (warp == 0) {
    if (elect_one()) {
      bool ok = true;
      int last_st = -1;
      uint32_t last_ph = 0;
      mbar_arrive_expect_tx(qdo_full, 2 * TILE_BYTES);
      tma_load_2d(sQ, &tmQ, qdo_full, h * HD, q0);
      tma_load_2d(sQ + CHUNK, &tmQ, qdo_full, h * HD + 64, q0);
      tma_load_2d(sDO, &tmDO, qdo_full, h * HD, q0);
      tma_load_2d(sDO + CHUNK, &tmDO, qdo_full, h * HD + 64, q0);
      for (int j = 0; j < n && ok; ++j) {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(&kv_empty[st], ph ^ 1u, status, 311)) { ok = false; break; }
        const int k0 = tile_at(j) * TK;
        uint8_t* k_dst = sKV + st * 2 * TILE_BYTES;
        uint8_t* v_dst = k_dst + TILE_BYTES;
        mbar_arrive_expect_tx(&kv_full[st], 2 * TILE_BYTES);
        tma_load_2d(k_dst, &tmK, &kv_full[st], kvh * HD, k0);
        tma_load_2d(k_dst + CHUNK, &tmK, &kv_full[st], kvh * HD + 64, k0);
        tma_load_2d(v_dst, &tmV, &kv_full[st], kvh * HD, k0);
        tma_load_2d(v_dst + CHUNK, &tmV, &kv_full[st], kvh * HD + 64, k0);
        last_st = st;
        last_ph = ph;
      }
      if (!ok && last_st >= 0) mbar_wait(&kv_full[last_st], last_ph, nullptr, 0);
      mbar_wait(qdo_full, 0, nullptr, 0);
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t ID_SS = idesc_bf16(TQ, TK, false, false);  // S, dP
      constexpr uint32_t ID_DQ = idesc_bf16(TQ, HD, false, true);   // dQ += dS K
      const uint32_t q_base = smem_u32(sQ), do_base = smem_u32(sDO);
      auto issue_s = [&](int j) {
        const uint32_t k_base = smem_u32(sKV + (j & 1) * 2 * TILE_BYTES);
        const uint32_t d = tS + (j & 1) * 128;
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * CHUNK + (kk & 3) * 32;
          mma_bf16_ss(d, sw128_desc(q_base + off, 16, 1024), sw128_desc(k_base + off, 16, 1024),
                      ID_SS, kk > 0 ? 1u : 0u);
        }
      };
      auto issue_dp = [&](int j) {
        const uint32_t v_base = smem_u32(sKV + (j & 1) * 2 * TILE_BYTES + TILE_BYTES);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * CHUNK + (kk & 3) * 32;
          mma_bf16_ss(tDP, sw128_desc(do_base + off, 16, 1024), sw128_desc(v_base + off, 16, 1024),
                      ID_SS, kk > 0 ? 1u : 0u);
        }
      };
      bool ok = mbar_wait(qdo_full, 0, status, 312);
      if (ok && n > 0) {
        ok = mbar_wait(&kv_full[0], 0, status, 313);
        if (ok) {
          tc_fence_after();
          issue_s(0);
          issue_dp(0);
          mma_commit(&s_full[0]);
        }
      }
      for (int j = 0; j < n && ok; ++j) {
        if (j + 1 < n) {
          if (!mbar_wait(&kv_full[(j + 1) & 1], ((j + 1) >> 1) & 1, status, 314)) { ok = false; break; }
          tc_fence_after();
          issue_s(j + 1);  // other S buffer: its dS(j-1) was consumed by dQ(j-1) before
          if (!mbar_wait(dp_free, j & 1, status, 315)) { ok = false; break; }
          tc_fence_after();
          issue_dp(j + 1);
          mma_commit(&s_full[(j + 1) & 1]);
        }
        if (!mbar_wait(ds_full, j & 1, status, 316)) { ok = false; break; }
        tc_fence_after();
        const uint32_t k_base = smem_u32(sKV + (j & 1) * 2 * TILE_BYTES);
        const uint32_t a = tS + (j & 1) * 128;
        // packed dS: the keys of softmax part p (columns [p C, p C + C), C = kKvCols)
        // in columns [p C, p C + C / 2)
        constexpr int steps = kKvCols / 16;
#pragma unroll
        for (int kk = 0; kk < TK / 16; ++kk)
          mma_bf16_ts(tDQ, a + (kk / steps) * kKvCols + (kk % steps) * 8,
                      sw128_desc(k_base + kk * 2048, CHUNK, 1024), ID_DQ,
                      (j > 0 || kk > 0) ? 1u : 0u);
        mma_commit(&kv_empty[j & 1]);
      }
      if (ok) mma_commit(dq_full);
    }
  } else {
    // ---------------- softmax warps (4 x kKvParts): query row per TMEM lane ----
    // part p owns key columns [p C, p C + C) and writes its packed dS into the first
    // C / 2 of them, which only it reads
    constexpr int C = kKvCols;
    const int quarter = warp & 3;
    const int part = (warp - 2) >> 2;
    const int cb = part * C;
    const int row = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const int s = q0 + row;
    const bool valid = s < g.S;
    int qi = -1, qd = 0;
    float l2 = 0.f, dl = 0.f;
    if (valid) {
      decode(g, s, qi, qd);
      l2 = lse[(int64_t)h * g.S + s] * kLog2e;
      dl = delta[(int64_t)h * g.S + s];
    }
    const int lo = qd > 0 ? g.a1 + (qi - g.a0) * g.km1 : 0;
    const float scale_log2 = scale * kLog2e;
    bool ok = true;
    for (int j = 0; j < n; ++j) {
      if (!mbar_wait(&s_full[j & 1], (j >> 1) & 1, status, 317)) { ok = false; break; }
      tc_fence_after();
      const uint32_t tSj = tS + (j & 1) * 128 + lane_off;
      float sv[C], dpv[C];
#pragma unroll
      for (int c = 0; c < C; c += 32) {
        tmem_ld32(tSj + cb + c, sv + c);
        tmem_ld32(tDP + lane_off + cb + c, dpv + c);
      }
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(dp_free);
      const int k0 = tile_at(j) * TK + cb;
      const bool full = k0 + C - 1 <= qi;
#pragma unroll
      for (int c0 = 0; c0 < C; c0 += 16) {
        uint32_t pk[8];
#pragma unroll
        for (int c = 0; c < 16; c += 2) {
          float dd[2];
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            const int ks = k0 + c0 + c + t;
            const bool allow = full || ks <= qi || (unsigned)(ks - lo) < (unsigned)qd;
            const float p = allow ? ex2_approx(sv[c0 + c + t] * scale_log2 - l2) : 0.f;
            dd[t] = p * (dpv[c0 + c + t] - dl);
          }
          pk[c / 2] = pack_bf16x2(dd[0], dd[1]);
        }
        tmem_st8(tSj + cb + c0 / 2, pk);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(ds_full);
    }
    if (ok && n > 0 && mbar_wait(dq_full, 0, status, 318)) {
      tc_fence_after();
#pragma unroll 1
      for (int c = cb; c < cb + C; c += 32) {
        float v[32];
        tmem_ld32(tDQ + lane_off + c, v);
        tmem_wait_ld();
        if (valid) {
          uint4* dst = reinterpret_cast<uint4*>(dq + (int64_t)s * dq_ss + h * HD + c);
#pragma unroll
          for (int u = 0; u < 4; ++u)
            dst[u] = make_uint4(pack_bf16x2(v[8 * u] * scale, v[8 * u + 1] * scale),
                                pack_bf16x2(v[8 * u + 2] * scale, v[8 * u + 3] * scale),
                                pack_bf16x2(v[8 * u + 4] * scale, v[8 * u + 5] * scale),
                                pack_bf16x2(v[8 * u + 6] * scale, v[8 * u + 7] * scale));
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

__global__ void __launch_bounds__(kKvThreads, 1)
attn_bwd_kv_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                   const float* __restrict__ lse, const float* __restrict__ delta,
                   float* __restrict__ dk_acc, float* __restrict__ dv_acc, PartGeom g, int Hkv,
                   int rep, float scale, int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sK = smem;
  uint8_t* sV = sK + TILE_BYTES;
  uint8_t* sQD = sV + TILE_BYTES;  // stage s: Q at + s * 2 * TILE, dO at + TILE
  float* sL = reinterpret_cast<float*>(sQD + 4 * TILE_BYTES);  // [2][TQ] lse * log2(e)
  float* sD = sL + 2 * TQ;                                       // [2][TQ] delta
  int* sA = reinterpret_cast<int*>(sD + 2 * TQ);                 // [2][TQ] query anchor
  int* sDp = sA + 2 * TQ;                                        // [2][TQ] query depth
  uint64_t* bars = reinterpret_cast<uint64_t*>(sDp + 2 * TQ);
  uint64_t* kv_full = bars + 0;
  uint64_t* qdo_full = bars + 1;   // [2]
  uint64_t* qdo_empty = bars + 3;  // [2]
  uint64_t* st_full = bars + 5;    // S^T(it) computed
  uint64_t* dpt_full = bars + 6;   // dP^T(it) computed
  uint64_t* p_full = bars + 7;     // P^T(it) written over S^T
  uint64_t* ds_full = bars + 8;    // dS^T(it) written over dP^T
  uint64_t* acc_full = bars + 9;
  uint64_t* meta_free = bars + 10;  // [2] per-query operands of a stage consumed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 12);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // grid (head, key tile): low key tiles are read by the most query tiles, and blocks
  // dispatch head-fastest, so the heaviest tiles of every head start first
  const int kt = blockIdx.y;
  const int h = blockIdx.x;
  const int kvh = h / rep;
  const int k0 = kt * TK;
  const Ranges qr = query_tiles(g, k0);
  const int n_it = qr.count();

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&qdo_full[i], 1);
      mbar_init(&qdo_empty[i], 1);
      mbar_init(&meta_free[i], 4 * kKvParts);
    }
    mbar_init(st_full, 1);
    mbar_init(dpt_full, 1);
    mbar_init(p_full, 4 * kKvParts);
    mbar_init(ds_full, 4 * kKvParts);
    mbar_init(acc_full, 1);
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
  const uint32_t tDK = tmem, tDV = tmem + 128, tS = tmem + 256, tDP = tmem + 384;

  if (warp == 0) {
    // TMA of K, V and the Q / dO ring; the whole warp stages each query tile's
    // (lse, delta, anchor, depth) once it may overwrite that stage's copy
    bool ok = true;
    int last_st = -1;
    uint32_t last_ph = 0;
    if (elect_one()) {
      mbar_arrive_expect_tx(kv_full, 2 * TILE_BYTES);
      tma_load_2d(sK, &tmK, kv_full, kvh * HD, k0);
      tma_load_2d(sK + CHUNK, &tmK, kv_full, kvh * HD + 64, k0);
      tma_load_2d(sV, &tmV, kv_full, kvh * HD, k0);
      tma_load_2d(sV + CHUNK, &tmV, kv_full, kvh * HD + 64, k0);
    }
    __syncwarp();
    for (int it = 0; it < n_it && ok; ++it) {
      const int st = it & 1;
      const uint32_t ph = (it >> 1) & 1;
      const int q0 = qr.at(it) * TQ;
      // per-query operands: lanes cover the tile's 128 queries, 4 each
      if (!mbar_wait(&meta_free[st], ph ^ 1u, status, 320)) { ok = false; }
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int r = u * 32 + lane;
        const int q = q0 + r;
        float lv = INFINITY, dl = 0.f;
        int qa = -1, qd = 0;
        if (q < g.S) {
          lv = lse[(int64_t)h * g.S + q] * kLog2e;
          dl = delta[(int64_t)h * g.S + q];
          decode(g, q, qa, qd);
        }
        sL[st * TQ + r] = lv;
        sD[st * TQ + r] = dl;
        sA[st * TQ + r] = qa;
        sDp[st * TQ + r] = qd;
      }
      __syncwarp();
      if (elect_one()) {
        // the stage's shared-memory operand writes precede the consumers' waits
        if (!mbar_wait(&qdo_empty[st], ph ^ 1u, status, 321)) ok = false;
        if (ok) {
          uint8_t* q_dst = sQD + st * 2 * TILE_BYTES;
          uint8_t* do_dst = q_dst + TILE_BYTES;
          mbar_arrive_expect_tx(&qdo_full[st], 2 * TILE_BYTES);  // release: covers sL..sDp
          tma_load_2d(q_dst, &tmQ, &qdo_full[st], h * HD, q0);
          tma_load_2d(q_dst + CHUNK, &tmQ, &qdo_full[st], h * HD + 64, q0);
          tma_load_2d(do_dst, &tmDO, &qdo_full[st], h * HD, q0);
          tma_load_2d(do_dst + CHUNK, &tmDO, &qdo_full[st], h * HD + 64, q0);
          last_st = st;
          last_ph = ph;
        }
      }
      ok = __all_sync(0xffffffffu, ok);
    }
    if (elect_one()) {
      mbar_wait(kv_full, 0, nullptr, 0);
      if (last_st >= 0) mbar_wait(&qdo_full[last_st], last_ph, nullptr, 0);
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t ID_KK = idesc_bf16(TK, TQ, false, false);  // S^T, dP^T
      constexpr uint32_t ID_KM = idesc_bf16(TK, HD, false, true);   // dV, dK (A from TMEM)
      const uint32_t k_base = smem_u32(sK), v_base = smem_u32(sV);
      auto issue_st = [&](int it) {
        const uint32_t q_base = smem_u32(sQD + (it & 1) * 2 * TILE_BYTES);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * CHUNK + (kk & 3) * 32;
          mma_bf16_ss(tS, sw128_desc(k_base + off, 16, 1024), sw128_desc(q_base + off, 16, 1024),
                      ID_KK, kk > 0 ? 1u : 0u);
        }
      };
      auto issue_dpt = [&](int it) {
        const uint32_t do_base = smem_u32(sQD + (it & 1) * 2 * TILE_BYTES) + TILE_BYTES;
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * CHUNK + (kk & 3) * 32;
          mma_bf16_ss(tDP, sw128_desc(v_base + off, 16, 1024), sw128_desc(do_base + off, 16, 1024),
                      ID_KK, kk > 0 ? 1u : 0u);
        }
      };
      // packed P^T / dS^T: the queries of compute part p (columns [p C, p C + C),
      // C = kKvCols) in columns [p C, p C + C / 2)
      auto a_col = [](int kk) {
        constexpr int steps = kKvCols / 16;  // 16-query K steps per part
        return (uint32_t)((kk / steps) * kKvCols + (kk % steps) * 8);
      };
      bool ok = mbar_wait(kv_full, 0, status, 322);
      if (ok && n_it > 0) {
        ok = mbar_wait(&qdo_full[0], 0, status, 323);
        if (ok) {
          tc_fence_after();
          issue_st(0);
          mma_commit(st_full);
          issue_dpt(0);
          mma_commit(dpt_full);
        }
      }
      for (int it = 0; it < n_it && ok; ++it) {
        const uint32_t q_base = smem_u32(sQD + (it & 1) * 2 * TILE_BYTES);
        const uint32_t do_base = q_base + TILE_BYTES;
        const uint32_t acc = it > 0 ? 1u : 0u;
        const bool more = it + 1 < n_it;
        if (!mbar_wait(p_full, it & 1, status, 324)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < TQ / 16; ++kk)
          mma_bf16_ts(tDV, tS + a_col(kk), sw128_desc(do_base + kk * 2048, CHUNK, 1024), ID_KM,
                      (acc | kk) != 0 ? 1u : 0u);
        if (more) {
          // S^T of the next query tile overlaps the dS^T arithmetic of this one
          if (!mbar_wait(&qdo_full[(it + 1) & 1], ((it + 1) >> 1) & 1, status, 326)) { ok = false; break; }
          tc_fence_after();
          issue_st(it + 1);
          mma_commit(st_full);
        }
        if (!mbar_wait(ds_full, it & 1, status, 325)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < TQ / 16; ++kk)
          mma_bf16_ts(tDK, tDP + a_col(kk), sw128_desc(q_base + kk * 2048, CHUNK, 1024), ID_KM,
                      (acc | kk) != 0 ? 1u : 0u);
        mma_commit(&qdo_empty[it & 1]);
        if (more) {
          issue_dpt(it + 1);  // after dK of this tile read dS^T (in-order tcgen05)
          mma_commit(dpt_full);
        }
      }
      if (ok) mma_commit(acc_full);
    }
  } else {
    // ---------------- compute warps (4 x kKvParts): thread = key row (TMEM lane) ----
    // part p owns query columns [p C, p C + C) and writes its packed P^T / dS^T into
    // the first C / 2 of those columns, which only it reads
    constexpr int C = kKvCols;
    const int quarter = warp & 3;
    const int part = (warp - 2) >> 2;
    const int cb = part * C;
    const int row = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const int kj = k0 + row;
    const bool kvalid = kj < g.S;
    int ka = 0, ke = 0;
    if (kvalid) decode(g, kj, ka, ke);
    const float scale_log2 = scale * kLog2e;
    bool ok = true;
    for (int it = 0; it < n_it; ++it) {
      const int q0 = qr.at(it) * TQ;
      const int buf = it & 1;
      const bool full = tile_fully_allowed(g, q0, k0);
      // ---- P^T = 2^(S^T c - lse') ----
      // the stage's per-query operands were written before its TMA was armed
      if (!mbar_wait(&qdo_full[buf], (it >> 1) & 1, status, 330)) { ok = false; break; }
      if (!mbar_wait(st_full, it & 1, status, 327)) { ok = false; break; }
      tc_fence_after();
      float pv[C];
#pragma unroll
      for (int c = 0; c < C; c += 32) tmem_ld32(tS + lane_off + cb + c, pv + c);
      tmem_wait_ld();
      if (full) {
        const float4* L4 = reinterpret_cast<const float4*>(sL + buf * TQ + cb);
#pragma unroll
        for (int c = 0; c < C; c += 4) {
          const float4 l4 = L4[c / 4];
          pv[c] = ex2_approx(pv[c] * scale_log2 - l4.x);
          pv[c + 1] = ex2_approx(pv[c + 1] * scale_log2 - l4.y);
          pv[c + 2] = ex2_approx(pv[c + 2] * scale_log2 - l4.z);
          pv[c + 3] = ex2_approx(pv[c + 3] * scale_log2 - l4.w);
        }
      } else {
        const float* L = sL + buf * TQ + cb;
        const int* QA = sA + buf * TQ + cb;
        const int* QD = sDp + buf * TQ + cb;
#pragma unroll
        for (int c = 0; c < C; ++c) {
          const int qa = QA[c];
          const bool allow =
              kvalid && qa >= 0 && (ke == 0 ? (ka <= qa) : (ka == qa && ke <= QD[c]));
          pv[c] = allow ? ex2_approx(pv[c] * scale_log2 - L[c]) : 0.f;
        }
      }
#pragma unroll
      for (int c0 = 0; c0 < C; c0 += 16) {
        uint32_t pw[8];
#pragma unroll
        for (int c = 0; c < 16; c += 2) pw[c / 2] = pack_bf16x2(pv[c0 + c], pv[c0 + c + 1]);
        tmem_st8(tS + lane_off + cb + c0 / 2, pw);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
      // ---- dS^T = P^T (dP^T - delta) ----
      if (!mbar_wait(dpt_full, it & 1, status, 328)) { ok = false; break; }
      tc_fence_after();
      const float4* D4 = reinterpret_cast<const float4*>(sD + buf * TQ + cb);
      // 16 columns at a time: packed dS^T for columns [c0, c0 + 16) lands in packed
      // columns [c0 / 2, c0 / 2 + 8), which this thread has already read
#pragma unroll
      for (int c0 = 0; c0 < C; c0 += 16) {
        float dv[16];
        tmem_ld16(tDP + lane_off + cb + c0, dv);
        tmem_wait_ld();
        uint32_t pw[8];
#pragma unroll
        for (int c = 0; c < 16; c += 4) {
          const float4 d4 = D4[(c0 + c) / 4];
          pw[c / 2] = pack_bf16x2(pv[c0 + c] * (dv[c] - d4.x), pv[c0 + c + 1] * (dv[c + 1] - d4.y));
          pw[c / 2 + 1] =
              pack_bf16x2(pv[c0 + c + 2] * (dv[c + 2] - d4.z), pv[c0 + c + 3] * (dv[c + 3] - d4.w));
        }
        tmem_st8(tDP + lane_off + cb + c0 / 2, pw);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(ds_full);
        mbar_arrive(&meta_free[buf]);
      }
    }
    // this head's dK, dV tile (key row per TMEM lane) -> the KV head's fp32 accumulators
    if (ok && n_it > 0 && mbar_wait(acc_full, 0, status, 329)) {
      tc_fence_after();
      const int64_t kv_ld = (int64_t)Hkv * HD;
#pragma unroll 1
      for (int c0 = cb; c0 < cb + C; c0 += 32) {
        float v[32];
        tmem_ld32(tDK + lane_off + c0, v);
        tmem_wait_ld();
        if (kvalid) atomic_add_row32(dk_acc + (int64_t)kj * kv_ld + kvh * HD + c0, v, 1.f);
        tmem_ld32(tDV + lane_off + c0, v);
        tmem_wait_ld();
        if (kvalid) atomic_add_row32(dv_acc + (int64_t)kj * kv_ld + kvh * HD + c0, v, 1.f);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// first stacked row of each segment of a launch group (row0[n] = total rows)
struct SegRows {
  int n;
  int row0[kMaxSeg + 1];
};

// delta (fp32, one [Hq, S_seg] block per segment at element Hq * row0_seg) =
// sum_d dO * O per (stacked row, head); zero the dQ accumulator row (when given) and,
// for the first Hkv heads, the dK / dV accumulator rows; zero the two work counters.
// Sixteen threads per (row, head), each reading 16 bytes of O and of dO.
__global__ void attn_bwd_prep_kernel(const __grid_constant__ SegRows sr, int Hq, int Hkv,
                                     const __nv_bfloat16* __restrict__ o, int64_t o_ss,
                                     const __nv_bfloat16* __restrict__ dout, int64_t do_ss,
                                     float* __restrict__ delta, float* __restrict__ dq_acc,
                                     float* __restrict__ dk_acc, float* __restrict__ dv_acc,
                                     int* __restrict__ counter) {
  if (blockIdx.x == 0 && threadIdx.x < 2) counter[threadIdx.x] = 0;  // dK/dV, dQ kernels
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t pair = t >> 4;  // (stacked row, head), heads fastest
  const int sub = threadIdx.x & 15;
  if (pair >= (int64_t)sr.row0[sr.n] * Hq) return;
  const int s = (int)(pair / Hq), h = (int)(pair - (int64_t)s * Hq);
  int sg = 0;
  while (sg + 1 < sr.n && s >= sr.row0[sg + 1]) ++sg;
  const int r0 = sr.row0[sg], S = sr.row0[sg + 1] - r0;
  const uint4 a = *reinterpret_cast<const uint4*>(o + (int64_t)s * o_ss + h * HD + sub * 8);
  const uint4 b = *reinterpret_cast<const uint4*>(dout + (int64_t)s * do_ss + h * HD + sub * 8);
  const __nv_bfloat162* a2 = reinterpret_cast<const __nv_bfloat162*>(&a);
  const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&b);
  float acc = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 x = __bfloat1622float2(a2[i]), y = __bfloat1622float2(b2[i]);
    acc = fmaf(x.x, y.x, acc);
    acc = fmaf(x.y, y.y, acc);
  }
#pragma unroll
  for (int m = 8; m > 0; m >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, m);
  if (sub == 0) delta[(int64_t)Hq * r0 + (int64_t)h * S + (s - r0)] = acc;
  const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
  if (dq_acc) {
    float4* d = reinterpret_cast<float4*>(dq_acc + (int64_t)s * Hq * HD + h * HD) + sub * 2;
    d[0] = z;
    d[1] = z;
  }
  if (h < Hkv) {
    float4* dk4 = reinterpret_cast<float4*>(dk_acc + (int64_t)s * Hkv * HD + h * HD) + sub * 2;
    float4* dv4 = reinterpret_cast<float4*>(dv_acc + (int64_t)s * Hkv * HD + h * HD) + sub * 2;
    dk4[0] = z;
    dk4[1] = z;
    dv4[0] = z;
    dv4[1] = z;
  }
}

// out (bf16, row stride ld) = mul * acc ([S, cols] fp32, contiguous)
__global__ void attn_cast_kernel(int S, int cols, const float* __restrict__ acc, float mul,
                                 __nv_bfloat16* __restrict__ out, int64_t ld) {
  const int64_t total = (int64_t)S * cols / 8;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = i * 8;
    const int64_t s = e / cols, c = e - s * cols;
    const float4 x = reinterpret_cast<const float4*>(acc + e)[0];
    const float4 y = reinterpret_cast<const float4*>(acc + e)[1];
    *reinterpret_cast<uint4*>(out + s * ld + c) =
        make_uint4(pack_bf16x2(x.x * mul, x.y * mul), pack_bf16x2(x.z * mul, x.w * mul),
                   pack_bf16x2(y.x * mul, y.y * mul), pack_bf16x2(y.z * mul, y.w * mul));
  }
}

// out (bf16) = mul * acc rounded to bf16, then every 128-wide head rotated back by the
// transpose of the rotary embedding with the row's cos / sin (cs: [S] rows of
// [cos 64 | sin 64], row stride cs_ld): one thread per (row, head, 8 pairs)
__global__ void attn_cast_rope_kernel(int S, int heads, const float* __restrict__ acc, float mul,
                                      __nv_bfloat16* __restrict__ out, int64_t ld,
                                      const __nv_bfloat16* __restrict__ cs, int64_t cs_ld) {
  const int64_t total = (int64_t)S * heads * 8;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t s = i / (heads * 8);
    const int r = (int)(i - s * heads * 8);
    const int h = r >> 3, p0 = (r & 7) * 8;
    const float* a = acc + (s * heads + h) * HD + p0;
    float va[8], vb[8], c[8], sn[8];
    const float4 a0 = reinterpret_cast<const float4*>(a)[0], a1 = reinterpret_cast<const float4*>(a)[1];
    const float4 b0 = reinterpret_cast<const float4*>(a + 64)[0];
    const float4 b1 = reinterpret_cast<const float4*>(a + 64)[1];
    va[0] = a0.x; va[1] = a0.y; va[2] = a0.z; va[3] = a0.w;
    va[4] = a1.x; va[5] = a1.y; va[6] = a1.z; va[7] = a1.w;
    vb[0] = b0.x; vb[1] = b0.y; vb[2] = b0.z; vb[3] = b0.w;
    vb[4] = b1.x; vb[5] = b1.y; vb[6] = b1.z; vb[7] = b1.w;
    load_bf16_f32<8>(cs + s * cs_ld + p0, c);
    load_bf16_f32<8>(cs + s * cs_ld + 64 + p0, sn);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      va[j] = rb16(va[j] * mul);
      vb[j] = rb16(vb[j] * mul);
      rope_rotate_pair(va[j], vb[j], c[j], sn[j], true);
    }
    __nv_bfloat16* o = out + s * ld + h * HD + p0;
    *reinterpret_cast<uint4*>(o) =
        make_uint4(pack_bf16x2(va[0], va[1]), pack_bf16x2(va[2], va[3]), pack_bf16x2(va[4], va[5]),
                   pack_bf16x2(va[6], va[7]));
    *reinterpret_cast<uint4*>(o + 64) =
        make_uint4(pack_bf16x2(vb[0], vb[1]), pack_bf16x2(vb[2], vb[3]), pack_bf16x2(vb[4], vb[5]),
                   pack_bf16x2(vb[6], vb[7]));
  }
}

int launch_cast_rope(int S, int heads, const float* acc, float mul, void* out, int64_t ld,
                     const void* cs, int64_t cs_ld, cudaStream_t st) {
  const int64_t total = (int64_t)S * heads * 8;
  int64_t blocks = (total + 255) / 256;
  if (blocks > (int64_t)sm_count() * 16) blocks = (int64_t)sm_count() * 16;
  attn_cast_rope_kernel<<<(unsigned)(blocks < 1 ? 1 : blocks), 256, 0, st>>>(
      S, heads, acc, mul, (__nv_bfloat16*)out, ld, (const __nv_bfloat16*)cs, cs_ld);
  PE_LAUNCHED();
  return PE_OK;
}

int launch_cast(int S, int cols, const float* acc, float mul, void* out, int64_t ld,
                cudaStream_t st) {
  const int64_t total = (int64_t)S * cols / 8;
  int64_t blocks = (total + 255) / 256;
  if (blocks > (int64_t)sm_count() * 16) blocks = (int64_t)sm_count() * 16;
  attn_cast_kernel<<<(unsigned)(blocks < 1 ? 1 : blocks), 256, 0, st>>>(
      S, cols, acc, mul, (__nv_bfloat16*)out, ld);
  PE_LAUNCHED();
  return PE_OK;
}

}  // namespace

bool attn_tc_bwd_ready() { return true; }

size_t attn_tc_bwd_acc_bytes(int64_t S, int Hq, int Hkv) {
  return (size_t)S * (Hq + 2 * Hkv) * HD * 4 + 256;  // + the work counter
}

int attn_bwd_tc_launch(int64_t S, int Hq, int Hkv, const void* q, int64_t q_ss, const void* k,
                       int64_t k_ss, const void* v, int64_t v_ss, const void* o, int64_t o_ss,
                       const void* dout, int64_t do_ss, const float* lse, void* dq,
                       int64_t dq_ss, void* dk, int64_t dk_ss, void* dv, int64_t dv_ss,
                       float* delta, float* acc, const MaskSpec& m, int* status,
                       cudaStream_t st, int variant) {
  PE_CHECK_ARG(o_ss % 8 == 0 && do_ss % 8 == 0 && dq_ss % 8 == 0 && dk_ss % 8 == 0 &&
                   dv_ss % 8 == 0 && al16(o) && al16(dout) && al16(dq) && al16(dk) && al16(dv),
               "attention backward (tcgen05): operands must be 16-byte aligned");
  CUtensorMap tq, tk, tv, tdo;
  int rc = make_tmap_2d(&tq, q, (uint64_t)Hq * HD, (uint64_t)S, (uint64_t)q_ss * 2, 64, TQ);
  if (!rc) rc = make_tmap_2d(&tk, k, (uint64_t)Hkv * HD, (uint64_t)S, (uint64_t)k_ss * 2, 64, TK);
  if (!rc) rc = make_tmap_2d(&tv, v, (uint64_t)Hkv * HD, (uint64_t)S, (uint64_t)v_ss * 2, 64, TK);
  if (!rc)
    rc = make_tmap_2d(&tdo, dout, (uint64_t)Hq * HD, (uint64_t)S, (uint64_t)do_ss * 2, 64, TQ);
  if (rc) return rc;
  const int Si = (int)S;
  float* dq_acc = acc;
  float* dk_acc = dq_acc + (int64_t)S * Hq * HD;
  float* dv_acc = dk_acc + (int64_t)S * Hkv * HD;
  int* counter = reinterpret_cast<int*>(dv_acc + (int64_t)S * Hkv * HD);
  PartGeom g{Si, (int)m.a0, (int)m.a1, m.kd - 1};
  if (variant == 0)
    return attn_bwd_tc_segments(1, &g, Hq, Hkv, q, q_ss, k, k_ss, v, v_ss, o, o_ss, dout, do_ss,
                                lse, dq, dq_ss, dk, dk_ss, dv, dv_ss, delta, dk_acc, nullptr, 0,
                                status, st);
  {
    SegRows sr{};
    sr.n = 1;
    sr.row0[1] = Si;
    const int64_t threads = (int64_t)Si * Hq * 16;
    attn_bwd_prep_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, st>>>(
        sr, Hq, Hkv, (const __nv_bfloat16*)o, o_ss, (const __nv_bfloat16*)dout, do_ss, delta,
        variant == 1 ? dq_acc : nullptr, dk_acc, dv_acc, counter);
    PE_LAUNCHED();
  }
  const float scale = 1.0f / sqrtf((float)HD);
  if (variant == 2) {
    {
      PE_CUDA_TRY(cudaFuncSetAttribute(attn_bwd_q_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)SMEM_BWD_Q));
      dim3 gq((unsigned)Hq, (unsigned)((S + TQ - 1) / TQ));
      attn_bwd_q_kernel<<<gq, kKvThreads, SMEM_BWD_Q, st>>>(tq, tk, tv, tdo, lse, delta,
                                                          (__nv_bfloat16*)dq, dq_ss, g, Hq / Hkv,
                                                          scale, status);
      PE_LAUNCHED();
    }
    {
      PE_CUDA_TRY(cudaFuncSetAttribute(attn_bwd_kv_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)SMEM_BWD_KV));
      dim3 gkv((unsigned)Hq, (unsigned)((S + TK - 1) / TK));
      attn_bwd_kv_kernel<<<gkv, kKvThreads, SMEM_BWD_KV, st>>>(tq, tk, tv, tdo, lse, delta,
                                                             dk_acc, dv_acc, g, Hkv, Hq / Hkv,
                                                             scale, status);
      PE_LAUNCHED();
    }
    rc = launch_cast(Si, Hkv * HD, dk_acc, scale, dk, dk_ss, st);
    if (!rc) rc = launch_cast(Si, Hkv * HD, dv_acc, 1.f, dv, dv_ss, st);
    return rc;
  }
  PE_CUDA_TRY(cudaFuncSetAttribute(attn_bwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)SMEM_BWD));
  dim3 grid((unsigned)Hq, (unsigned)((S + TK - 1) / TK));
  attn_bwd_tc_kernel<<<grid, kThreads, SMEM_BWD, st>>>(tq, tk, tv, tdo, lse, delta, dq_acc, dk_acc,
                                                       dv_acc, g, Hq, Hkv, Hq / Hkv, scale, status);
  PE_LAUNCHED();
  rc = launch_cast(Si, Hq * HD, dq_acc, scale, dq, dq_ss, st);
  if (!rc) rc = launch_cast(Si, Hkv * HD, dk_acc, scale, dk, dk_ss, st);
  if (!rc) rc = launch_cast(Si, Hkv * HD, dv_acc, 1.f, dv, dv_ss, st);
  return rc;
}

size_t attn_tc_seg_acc_bytes(int64_t rows, int Hkv) {
  return (size_t)rows * 2 * Hkv * HD * 4 + 256;  // dK, dV accumulators + the work counters
}

int attn_bwd_tc_segments(int nseg, const PartGeom* g, int Hq, int Hkv, const void* q,
                         int64_t q_ss, const void* k, int64_t k_ss, const void* v, int64_t v_ss,
                         const void* o, int64_t o_ss, const void* dout, int64_t do_ss,
                         const float* lse, void* dq, int64_t dq_ss, void* dk, int64_t dk_ss,
                         void* dv, int64_t dv_ss, float* delta, float* acc,
                         const void* rope_cs, int64_t cs_ld, int* status, cudaStream_t st) {
  PE_CHECK_ARG(o_ss % 8 == 0 && do_ss % 8 == 0 && dq_ss % 8 == 0 && dk_ss % 8 == 0 &&
                   dv_ss % 8 == 0 && al16(o) && al16(dout) && al16(dq) && al16(dk) && al16(dv),
               "attention backward (tcgen05): operands must be 16-byte aligned");
  PE_CHECK_ARG(!rope_cs || (cs_ld % 8 == 0 && cs_ld >= HD && al16(rope_cs)),
               "attention backward (tcgen05): the rotary table must be 16-byte aligned bf16 rows "
               "of at least head_dim entries");
  std::vector<int64_t> rows(nseg + 1, 0);
  for (int s = 0; s < nseg; ++s) rows[s + 1] = rows[s] + g[s].S;
  const float scale = 1.0f / sqrtf((float)HD);
  // every launch group reuses the accumulators from their start: its prep zeroes
  // them after the previous group's casts (stream order)
  for (auto [b, e] : seg_groups(nseg, g)) {
    const int64_t rb = rows[b], R = rows[e] - rows[b];
    PE_CHECK_ARG(R * Hq < (1ll << 31), "attention backward: too many stacked rows");
    float* dk_acc = acc;
    float* dv_acc = dk_acc + R * Hkv * HD;
    int* counter = reinterpret_cast<int*>(dv_acc + R * Hkv * HD);
    auto at = [rb](const void* p, int64_t ss) {
      return static_cast<const uint8_t*>(p) + rb * ss * 2;
    };
    auto at_mut = [rb](void* p, int64_t ss) { return static_cast<uint8_t*>(p) + rb * ss * 2; };
    const float* lse_g = lse + Hq * rb;
    float* delta_g = delta + Hq * rb;
    {
      SegRows sr{};
      sr.n = e - b;
      for (int s = b; s < e; ++s) sr.row0[s - b + 1] = (int)(rows[s + 1] - rb);
      const int64_t threads = R * Hq * 16;
      attn_bwd_prep_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, st>>>(
          sr, Hq, Hkv, (const __nv_bfloat16*)at(o, o_ss), o_ss,
          (const __nv_bfloat16*)at(dout, do_ss), do_ss, delta_g, nullptr, dk_acc, dv_acc,
          counter);
      PE_LAUNCHED();
    }
    const void* cs_g = rope_cs ? static_cast<const uint8_t*>(rope_cs) + rb * cs_ld * 2 : nullptr;
    int rc = attn_bwd_q2_launch(e - b, g + b, Hq, Hkv, at(q, q_ss), q_ss, at(k, k_ss), k_ss,
                                at(v, v_ss), v_ss, at(dout, do_ss), do_ss, lse_g, delta_g,
                                at_mut(dq, dq_ss), dq_ss, cs_g, cs_ld, counter + 1, status, st);
    if (!rc)
      rc = attn_bwd_kv2_launch(e - b, g + b, Hq, Hkv, at(q, q_ss), q_ss, at(k, k_ss), k_ss,
                               at(v, v_ss), v_ss, at(dout, do_ss), do_ss, lse_g, delta_g, dk_acc,
                               dv_acc, counter, status, st);
    if (!rc)
      rc = cs_g ? launch_cast_rope((int)R, Hkv, dk_acc, scale, at_mut(dk, dk_ss), dk_ss, cs_g, cs_ld, st)
                : launch_cast((int)R, Hkv * HD, dk_acc, scale, at_mut(dk, dk_ss), dk_ss, st);
    if (!rc) rc = launch_cast((int)R, Hkv * HD, dv_acc, 1.f, at_mut(dv, dv_ss), dv_ss, st);
    if (rc) return rc;
  }
  return PE_OK;
}

}  // namespace pe
