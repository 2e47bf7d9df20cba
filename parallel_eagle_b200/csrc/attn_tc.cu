// Cross-depth masked flash attention on the 5th-generation tensor cores
// (forward).  bf16 in/out, fp32 softmax, head_dim 128, partition slot layout
// (reference src/pe/nn.py:71-89 with the mask of src/pe/masks.py:43-61 and the
// segment layout of src/pe/partition.py:41-55).
//
// One CTA = one 128-slot query tile of one head.  The attend rule leaves each
// query row (anchor i, depth d) exactly two key intervals: the real keys
// [0, i] and its own anchor's prediction keys [lo_i, lo_i + d).  A query tile
// therefore visits only the key tiles under those intervals: the causal band of
// the real stream plus one or two tiles on the prediction-slot diagonal -- the
// ~90% of the dense (S x S) score matrix the rule forbids is never computed.
//
// Warp roles (320 threads):
//   warp 0      TMA: Q tile once, then K/V tiles into a 2-stage ring
//   warp 1      tcgen05.mma issue: S_j = Q K_j^T into a double-buffered TMEM
//               score tile, O += P_j V_j into the TMEM output tile
//   warps 2..9  softmax: two warps per TMEM lane quarter, each owning 64 of the
//               128 key columns (and 64 of the 128 output columns), so every
//               scheduler has two independent softmax warps to hide latency;
//               the pair exchanges its row maxima through shared memory
// TMEM: O [128 x 128 fp32] in columns 0..127, S buffers in 128..383.
#include "attn_tc.cuh"

namespace pe {
namespace {

using namespace sm100;
using namespace attn_tc;

constexpr int kThreads = 320;
constexpr int kSoftmaxThreads = 256;
constexpr size_t SMEM_FWD = 1024 + TILE_BYTES /*Q*/ + 2 * 2 * TILE_BYTES /*K,V x2*/ +
                            TILE_BYTES /*P*/ + 2 * 2 * TQ * 4 /*row max exchange*/ +
                            2 * TQ * 4 /*row sums*/ + 256;

// Key tiles visited by query tile qt: [0, r_end) then [m_beg, m_end) (may be empty)
struct TileList {
  int r_end, m_beg, m_end;
  __device__ __forceinline__ int count() const { return r_end + (m_end - m_beg); }
  __device__ __forceinline__ int tile(int j) const { return j < r_end ? j : m_beg + (j - r_end); }
};

__device__ __forceinline__ TileList tiles_for(const PartGeom& g, int q0) {
  const int last = min(q0 + TQ, g.S) - 1;
  int i_last, d_last;
  decode(g, last, i_last, d_last);
  // largest anchor in the tile: the last row's, or -- when the tile straddles the
  // real/prediction boundary -- the last real row's (anchor a1 - 1 at most)
  const int i_max = q0 < g.a1 ? max(i_last, min(last, g.a1 - 1)) : i_last;
  TileList L;
  L.r_end = i_max / TK + 1;
  L.m_beg = L.m_end = 0;
  if (last >= g.a1 && g.km1 > 0) {
    const int first = max(q0, g.a1);
    int i_first, d_first;
    decode(g, first, i_first, d_first);
    const int lo = g.a1 + (i_first - g.a0) * g.km1;
    const int hi = g.a1 + (i_last - g.a0 + 1) * g.km1;  // exclusive
    int mb = lo / TK, me = (hi - 1) / TK + 1;
    if (mb < L.r_end) mb = L.r_end;  // already covered by the real band
    if (me > mb) {
      L.m_beg = mb;
      L.m_end = me;
    }
  }
  return L;
}

__device__ __forceinline__ void named_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__global__ void __launch_bounds__(kThreads, 1)
attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, __nv_bfloat16* __restrict__ O,
                   int64_t o_ss, float* __restrict__ lse, PartGeom g, int Hq, int rep,
                   float scale_log2, int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sKV = sQ + TILE_BYTES;  // stage s: K at +s*2*TILE, V at +TILE
  uint8_t* sP = sKV + 4 * TILE_BYTES;
  float* sMax = reinterpret_cast<float*>(sP + TILE_BYTES);  // [tile parity][half][TQ]
  float* sSum = sMax + 2 * 2 * TQ;                          // [half][TQ]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sSum + 2 * TQ);
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 1;   // [2]
  uint64_t* kv_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;    // [2]
  uint64_t* s_empty = bars + 7;   // [2]
  uint64_t* p_full = bars + 9;
  uint64_t* pv_done = bars + 10;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 11);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_qt = (g.S + TQ - 1) / TQ;
  // grid (head, tile): blocks dispatch head-fastest, so the heaviest tiles of every
  // head start first
  const int qt = num_qt - 1 - (int)blockIdx.y;
  const int h = blockIdx.x;
  const int kvh = h / rep;
  const int q0 = qt * TQ;
  const TileList tl = tiles_for(g, q0);
  const int n = tl.count();

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 8);
    }
    mbar_init(p_full, 8);
    mbar_init(pv_done, 1);
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
  const uint32_t tO = tmem, tS0 = tmem + 128;

  if (warp == 0) {
    if (elect_one()) {
      bool ok = true;
      int last_st = -1;
      uint32_t last_ph = 0;
      mbar_arrive_expect_tx(q_full, TILE_BYTES);
      tma_load_2d(sQ, &tmQ, q_full, h * HD, q0);
      tma_load_2d(sQ + CHUNK, &tmQ, q_full, h * HD + 64, q0);
      for (int j = 0; j < n && ok; ++j) {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(&kv_empty[st], ph ^ 1u, status, 201)) { ok = false; break; }
        const int k0 = tl.tile(j) * TK;
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
      mbar_wait(q_full, 0, nullptr, 0);
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t IDESC_S = idesc_bf16(TQ, TK, false, false);
      constexpr uint32_t IDESC_O = idesc_bf16(TQ, HD, false, true);
      const uint32_t q_base = smem_u32(sQ), p_base = smem_u32(sP);
      bool ok = mbar_wait(q_full, 0, status, 202);
      auto issue_s = [&](int j) -> bool {
        const int st = j & 1;
        if (!mbar_wait(&kv_full[st], (j >> 1) & 1, status, 203)) return false;
        if (!mbar_wait(&s_empty[st], ((j >> 1) & 1) ^ 1u, status, 204)) return false;
        tc_fence_after();
        const uint32_t k_base = smem_u32(sKV + st * 2 * TILE_BYTES);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * CHUNK + (kk & 3) * 32;
          mma_bf16_ss(tS0 + st * 128, sw128_desc(q_base + off, 16, 1024),
                      sw128_desc(k_base + off, 16, 1024), IDESC_S, kk > 0 ? 1u : 0u);
        }
        mma_commit(&s_full[st]);
        return true;
      };
      if (ok && n > 0) ok = issue_s(0);
      for (int j = 0; j < n && ok; ++j) {
        if (j + 1 < n && !issue_s(j + 1)) { ok = false; break; }
        if (!mbar_wait(p_full, j & 1, status, 205)) { ok = false; break; }
        tc_fence_after();
        const int st = j & 1;
        const uint32_t v_base = smem_u32(sKV + st * 2 * TILE_BYTES + TILE_BYTES);
#pragma unroll
        for (int kk = 0; kk < TK / 16; ++kk) {
          const uint32_t poff = (kk >> 2) * CHUNK + (kk & 3) * 32;
          mma_bf16_ss(tO, sw128_desc(p_base + poff, 16, 1024),
                      sw128_desc(v_base + kk * 2048, CHUNK, 1024), IDESC_O,
                      (j > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(&kv_empty[st]);
        mma_commit(pv_done);
      }
    }
  } else {
    // ---------------- softmax warps: row (TMEM lane) x half of the columns ----------------
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;  // warps 2..5 -> 0, 6..9 -> 1
    const int cb = half * 64;          // key columns / output columns owned
    const int row = quarter * 32 + lane;
    const int s = q0 + row;
    const bool valid = s < g.S;
    int qi = 0, qd = 0;
    if (valid) decode(g, s, qi, qd);
    const int lo = qd > 0 ? g.a1 + (qi - g.a0) * g.km1 : 0;
    const int hi = lo + qd;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n; ++j) {
      const int st = j & 1;
      if (!mbar_wait(&s_full[st], (j >> 1) & 1, status, 206)) { ok = false; break; }
      tc_fence_after();
      float sc[64];
      tmem_ld32(tS0 + st * 128 + lane_off + cb, sc);
      tmem_ld32(tS0 + st * 128 + lane_off + cb + 32, sc + 32);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_empty[st]);
      const int k0 = tl.tile(j) * TK + cb;
      float mt = -INFINITY;
#pragma unroll
      for (int c = 0; c < 64; ++c) {
        const int kslot = k0 + c;
        const bool allow = (kslot <= qi) || (kslot >= lo && kslot < hi);
        sc[c] = allow ? sc[c] * scale_log2 : -INFINITY;
        mt = fmaxf(mt, sc[c]);
      }
      // combine the row maximum with the partner warp (other half of the columns)
      float* xm = sMax + (j & 1) * 2 * TQ;
      xm[half * TQ + row] = mt;
      named_sync(1, kSoftmaxThreads);
      mt = fmaxf(mt, xm[(half ^ 1) * TQ + row]);
      const float m_new = fmaxf(m, mt);
      const float m_use = m_new == -INFINITY ? 0.f : m_new;
      const float alpha = (m == m_new) ? 1.f : exp2f(m - m_use);
      float rs = 0.f;
      uint32_t pk[32];
#pragma unroll
      for (int c = 0; c < 64; c += 2) {
        const float p0 = exp2f(sc[c] - m_use), p1 = exp2f(sc[c + 1] - m_use);
        rs += p0 + p1;
        pk[c / 2] = pack_bf16x2(p0, p1);
      }
      l = l * alpha + rs;
      m = m_new;
      if (j > 0) {
        // O holds the sum over tiles < j: wait for PV(j-1) before touching O or P
        if (!mbar_wait(pv_done, (j - 1) & 1, status, 207)) { ok = false; break; }
        tc_fence_after();
        if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
          for (int c = 0; c < 64; c += 32) {
            float ov[32];
            tmem_ld32(tO + lane_off + cb + c, ov);
            tmem_wait_ld();
            uint32_t ou[32];
#pragma unroll
            for (int t = 0; t < 32; ++t) ou[t] = __float_as_uint(ov[t] * alpha);
            tmem_st16(tO + lane_off + cb + c, ou);
            tmem_st16(tO + lane_off + cb + c + 16, ou + 16);
          }
          tmem_wait_st();
        }
      }
      // this half's 64 keys of the P row -> shared memory (one 128B-swizzled chunk)
      uint8_t* base = sP + half * CHUNK;
#pragma unroll
      for (int u = 0; u < 8; ++u)
        *reinterpret_cast<uint4*>(base + swz(row, u)) =
            make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
      fence_proxy_async();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    // row sums: each half accumulated its own columns
    sSum[half * TQ + row] = l;
    named_sync(1, kSoftmaxThreads);
    l += sSum[(half ^ 1) * TQ + row];
    if (ok && n > 0 && mbar_wait(pv_done, (n - 1) & 1, status, 208)) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll 1
      for (int c = 0; c < 64; c += 32) {
        float ov[32];
        tmem_ld32(tO + lane_off + cb + c, ov);
        tmem_wait_ld();
        if (valid) {
          uint4* dst = reinterpret_cast<uint4*>(O + (int64_t)s * o_ss + h * HD + cb + c);
#pragma unroll
          for (int q = 0; q < 4; ++q)
            dst[q] = make_uint4(pack_bf16x2(ov[8 * q] * inv, ov[8 * q + 1] * inv),
                                pack_bf16x2(ov[8 * q + 2] * inv, ov[8 * q + 3] * inv),
                                pack_bf16x2(ov[8 * q + 4] * inv, ov[8 * q + 5] * inv),
                                pack_bf16x2(ov[8 * q + 6] * inv, ov[8 * q + 7] * inv));
        }
      }
      if (valid && half == 0) lse[(int64_t)h * g.S + s] = (m + log2f(l)) * kLn2;
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
// Two query tiles per CTA (rows q0 .. q0 + 255 of one head), so the tensor core
// always has one tile's MMAs to run while the other tile's softmax executes:
//
//   warp 0      TMA: both Q tiles once, then K/V tiles into a 2-stage ring
//   warp 1      MMA issue, per key tile j:  PV_A(j-1) S_A(j) PV_B(j-1) S_B(j)
//               (S_t = Q_t K^T into TMEM; PV_t: O_t += P_t V with P_t read from
//               TMEM -- the tcgen05 A-from-TMEM form -- so P never touches
//               shared memory)
//   warps 2..3  idle (they complete warpgroup 0, whose registers go to the softmax)
//   warps 4..7  softmax of tile A, one thread per query row (TMEM lane)
//   warps 8..11 softmax of tile B
//
// Warpgroup 0 (TMA, MMA) drops to 56 registers per thread and the two softmax
// warpgroups rise to 224, enough to hold a full 128-score row plus the packed
// probabilities without spilling (the CTA launches with 384 x 168).
//
// TMEM: O_A cols 0..127, O_B 128..255, S_A 256..383, S_B 384..511; P_t is
// written as packed bf16 pairs over the first 64 columns of S_t.
//
// The CTA walks the union of both tiles' key-tile lists; for a key tile one of
// the tiles does not need, that tile's MMAs are skipped (its barriers still
// advance, keeping every role in lockstep).  The running row maximum is only
// raised (and O rescaled) when it grows by more than 2^8: until then
// P = 2^(x - m) <= 256 against the stale maximum, and O and the row sum stay
// consistent because both are relative to the same m.
// ------------------------------------------------------------------------ //
constexpr int kThreads2 = 384;
constexpr int kRegsLow = 56, kRegsHigh = 224;  // 128 x 56 + 256 x 224 = 384 x 168
constexpr size_t SMEM_FWD2 = 1024 + 2 * TILE_BYTES /*Q_A, Q_B*/ + 2 * 2 * TILE_BYTES /*K,V x2*/ + 256;
constexpr float kRescaleLog2 = 8.f;
// one pair of scores in EMU takes its exponential from the FMA-pipe polynomial (0:
// all on the SFU); the SFU alone runs one exp per score, which at head_dim 128 takes
// as long as the tile's two MMAs.  The kernel is instantiated for a few ratios
// (attn_fwd_tc_segments' `emu`); kEmuDefault is the one the step uses.
constexpr int kEmuDefault = 4;

struct PairTiles {
  TileList a, b;  // b empty (count 0) when the second query tile lies past the sequence
  __device__ __forceinline__ static bool in(const TileList& l, int t) {
    return t < l.r_end || (t >= l.m_beg && t < l.m_end);
  }
  __device__ __forceinline__ bool use_a(int t) const { return in(a, t); }
  __device__ __forceinline__ bool use_b(int t) const { return in(b, t); }
  // smallest key tile > t that either query tile visits, or -1
  __device__ __forceinline__ int next(int t) const {
    int best = 0x7fffffff;
    auto cand = [&](int lo, int hi) {
      const int c = max(t + 1, lo);
      if (c < hi && c < best) best = c;
    };
    cand(0, max(a.r_end, b.r_end));
    cand(a.m_beg, a.m_end);
    cand(b.m_beg, b.m_end);
    return best == 0x7fffffff ? -1 : best;
  }
};

template <int kEmuEvery>
__global__ void __launch_bounds__(kThreads2, 1)
attn_fwd_tc2_kernel(const __grid_constant__ SegTable tab, __nv_bfloat16* __restrict__ O,
                    int64_t o_ss, float* __restrict__ lse, int Hq, int rep, float scale_log2,
                    int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sQ = smem;                  // tile t at + t * TILE_BYTES
  uint8_t* sKV = sQ + 2 * TILE_BYTES;  // stage s: K at + s * 2 * TILE, V at + TILE
  uint64_t* bars = reinterpret_cast<uint64_t*>(sKV + 4 * TILE_BYTES);
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 1;   // [2]
  uint64_t* kv_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;    // [query tile]
  uint64_t* p_full = bars + 7;    // [query tile]
  uint64_t* o_full = bars + 9;    // [query tile]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 11);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // grid (head, unit): blocks dispatch head-fastest, so the heaviest pairs of every
  // head start first -- stacked segments in the work list's order, a lone segment
  // from its last pair down
  int sg, pr;
  if (tab.nwork > 0) {
    unpack_work(tab.work[blockIdx.y], sg, pr);
  } else {
    sg = 0;
    pr = (tab.g[0].S + 2 * TQ - 1) / (2 * TQ) - 1 - (int)blockIdx.y;
  }
  const PartGeom g = tab.g[sg];
  const CUtensorMap* tmQ = &tab.tm[sg][0];
  const CUtensorMap* tmK = &tab.tm[sg][1];
  const CUtensorMap* tmV = &tab.tm[sg][2];
  O += (int64_t)tab.row0[sg] * o_ss;
  lse += (int64_t)Hq * tab.row0[sg];
  const int h = blockIdx.x;
  const int kvh = h / rep;
  const int q0 = pr * 2 * TQ;
  PairTiles pt;
  pt.a = tiles_for(g, q0);
  if (q0 + TQ < g.S) {
    pt.b = tiles_for(g, q0 + TQ);
  } else {
    pt.b.r_end = pt.b.m_beg = pt.b.m_end = 0;
  }

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
      mbar_init(&o_full[i], 1);
    }
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
  if (warp < 4) {
    setmaxnreg_dec<kRegsLow>();
    if (warp == 0) {
      if (elect_one()) {
        bool ok = true;
        int last_st = -1;
        uint32_t last_ph = 0;
        mbar_arrive_expect_tx(q_full, 2 * TILE_BYTES);
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          tma_load_2d(sQ + t * TILE_BYTES, tmQ, q_full, h * HD, q0 + t * TQ);
          tma_load_2d(sQ + t * TILE_BYTES + CHUNK, tmQ, q_full, h * HD + 64, q0 + t * TQ);
        }
        int j = 0;
        for (int kt = 0; kt >= 0 && ok; kt = pt.next(kt), ++j) {
          const int st = j & 1;
          const uint32_t ph = (j >> 1) & 1;
          if (!mbar_wait(&kv_empty[st], ph ^ 1u, status, 211)) { ok = false; break; }
          const int k0 = kt * TK;
          uint8_t* k_dst = sKV + st * 2 * TILE_BYTES;
          uint8_t* v_dst = k_dst + TILE_BYTES;
          mbar_arrive_expect_tx(&kv_full[st], 2 * TILE_BYTES);
          tma_load_2d(k_dst, tmK, &kv_full[st], kvh * HD, k0);
          tma_load_2d(k_dst + CHUNK, tmK, &kv_full[st], kvh * HD + 64, k0);
          tma_load_2d(v_dst, tmV, &kv_full[st], kvh * HD, k0);
          tma_load_2d(v_dst + CHUNK, tmV, &kv_full[st], kvh * HD + 64, k0);
          last_st = st;
          last_ph = ph;
        }
        if (!ok && last_st >= 0) mbar_wait(&kv_full[last_st], last_ph, nullptr, 0);
        mbar_wait(q_full, 0, nullptr, 0);
      }
    } else if (warp == 1) {
      if (elect_one()) {
        constexpr uint32_t IDESC_S = idesc_bf16(TQ, TK, false, false);
        constexpr uint32_t IDESC_O = idesc_bf16(TQ, HD, false, true);
        bool ok = mbar_wait(q_full, 0, status, 212);
        auto issue_s = [&](int t, int st) {
          const uint32_t q_base = smem_u32(sQ + t * TILE_BYTES);
          const uint32_t k_base = smem_u32(sKV + st * 2 * TILE_BYTES);
          const uint32_t d = tmem + 256 + t * 128;
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk) {
            const uint32_t off = (kk >> 2) * CHUNK + (kk & 3) * 32;
            mma_bf16_ss(d, sw128_desc(q_base + off, 16, 1024), sw128_desc(k_base + off, 16, 1024),
                        IDESC_S, kk > 0 ? 1u : 0u);
          }
        };
        auto issue_pv = [&](int t, int st, bool first) {
          const uint32_t v_base = smem_u32(sKV + st * 2 * TILE_BYTES + TILE_BYTES);
          const uint32_t p = tmem + 256 + t * 128;
#pragma unroll
          for (int kk = 0; kk < TK / 16; ++kk)
            mma_bf16_ts(tmem + t * 128, p + kk * 8, sw128_desc(v_base + kk * 2048, CHUNK, 1024),
                        IDESC_O, (!first || kk > 0) ? 1u : 0u);
        };
        // step 0: S of both tiles for key tile 0 (every query row sees key 0)
        if (ok) ok = mbar_wait(&kv_full[0], 0, status, 213);
        if (ok) {
          tc_fence_after();
          issue_s(0, 0);
          mma_commit(&s_full[0]);
          if (pt.use_b(0)) issue_s(1, 0);
          mma_commit(&s_full[1]);
        }
        bool pv_a = false, pv_b = false;
        int j = 0;
        for (int kt = 0; kt >= 0 && ok; ++j) {
          const int st = j & 1;
          const int kn = pt.next(kt);
          const int stn = (j + 1) & 1;
          // tile A: PV of key tile kt, then S of the next key tile
          if (!mbar_wait(&p_full[0], j & 1, status, 214)) { ok = false; break; }
          tc_fence_after();
          if (pt.use_a(kt)) {
            issue_pv(0, st, !pv_a);
            pv_a = true;
          }
          if (kn >= 0) {
            if (!mbar_wait(&kv_full[stn], ((j + 1) >> 1) & 1, status, 215)) { ok = false; break; }
            tc_fence_after();
            if (pt.use_a(kn)) issue_s(0, stn);
            mma_commit(&s_full[0]);
          }
          // tile B
          if (!mbar_wait(&p_full[1], j & 1, status, 216)) { ok = false; break; }
          tc_fence_after();
          if (pt.use_b(kt)) {
            issue_pv(1, st, !pv_b);
            pv_b = true;
          }
          if (kn >= 0) {
            if (pt.use_b(kn)) issue_s(1, stn);
            mma_commit(&s_full[1]);
          }
          mma_commit(&kv_empty[st]);
          kt = kn;
        }
        if (ok) {
          mma_commit(&o_full[0]);
          mma_commit(&o_full[1]);
        }
      }
    }
  } else {
    setmaxnreg_inc<kRegsHigh>();
    // ---------------- softmax: warps 4..7 tile A, 8..11 tile B; thread = query row ----
    const int t = (warp - 4) >> 2;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const int s = q0 + t * TQ + row;
    const bool valid = s < g.S;
    int qi = -1, qd = 0;
    if (valid) decode(g, s, qi, qd);
    const int lo = qd > 0 ? g.a1 + (qi - g.a0) * g.km1 : 0;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t tS = tmem + 256 + t * 128 + lane_off;
    const uint32_t tO = tmem + t * 128 + lane_off;
    const TileList& mine = t == 0 ? pt.a : pt.b;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    int j = 0;
    for (int kt = 0; kt >= 0; kt = pt.next(kt), ++j) {
      if (!mbar_wait(&s_full[t], j & 1, status, 217)) { ok = false; break; }
      tc_fence_after();
      if (PairTiles::in(mine, kt)) {
        float x[128];
#pragma unroll
        for (int c = 0; c < 128; c += 32) tmem_ld32(tS + c, x + c);
        tmem_wait_ld();
        const int k0 = kt * TK;
        if (k0 + TK - 1 > qi) {  // not every key is a real key <= the row's anchor: mask
#pragma unroll
          for (int c = 0; c < 128; ++c) {
            const int ks = k0 + c;
            const bool allow = ks <= qi || (unsigned)(ks - lo) < (unsigned)qd;
            x[c] = allow ? x[c] : -INFINITY;
          }
        }
        // maximum of the raw scores (the scale is positive, so it commutes with the
        // maximum): 4 independent chains of 3-input maxima
        float mp[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) mp[u] = -INFINITY;
#pragma unroll
        for (int c = 0; c < 128; c += 8) {
#pragma unroll
          for (int u = 0; u < 4; ++u) mp[u] = max3f(mp[u], x[c + 2 * u], x[c + 2 * u + 1]);
        }
        const float mt = max3f(mp[0], mp[1], fmaxf(mp[2], mp[3])) * scale_log2;
        // raise the reference maximum only when the tile exceeds it by > 2^8
        float alpha = 1.f;
        if (mt > m + kRescaleLog2) {
          alpha = m == -INFINITY ? 0.f : ex2_approx(m - mt);
          m = mt;
          l *= alpha;
        }
        const float nm = m == -INFINITY ? 0.f : -m;
        // P_t = 2^(x c - m) over the first 64 columns of S_t (packed bf16 pairs): the
        // scale-and-subtract and the 4 partial row sums run as packed f32x2 operations,
        // and every kEmuEvery-th pair's exponential runs on the FMA pipe
        float2 rs[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) rs[u] = make_float2(0.f, 0.f);
        const float2 sc = make_float2(scale_log2, scale_log2), off = make_float2(nm, nm);
#pragma unroll
        for (int c0 = 0; c0 < 128; c0 += 32) {
          uint32_t pk[16];
#pragma unroll
          for (int c = 0; c < 32; c += 2) {
            const float2 y = fma2(make_float2(x[c0 + c], x[c0 + c + 1]), sc, off);
            float2 p;
            if (kEmuEvery > 0 && (c / 2) % kEmuEvery == kEmuEvery - 1) {
              p = exp2_poly2(y);
            } else {
              p.x = ex2_approx(y.x);
              p.y = ex2_approx(y.y);
            }
            rs[(c >> 1) & 3] = add2(rs[(c >> 1) & 3], p);
            pk[c / 2] = pack_bf16x2(p.x, p.y);
          }
          tmem_st16(tS + c0 / 2, pk);
        }
        const float2 rsum = add2(add2(rs[0], rs[1]), add2(rs[2], rs[3]));
        l += rsum.x + rsum.y;
        // O holds the tiles before this one (their PV completed before this S did):
        // rescale it when the maximum moved
        if (__any_sync(0xffffffffu, alpha != 1.f) && j > 0) {
#pragma unroll 1
          for (int c = 0; c < 128; c += 32) {
            float ov[32];
            tmem_ld32(tO + c, ov);
            tmem_wait_ld();
            uint32_t ou[32];
#pragma unroll
            for (int u = 0; u < 32; ++u) ou[u] = __float_as_uint(ov[u] * alpha);
            tmem_st32(tO + c, ou);
          }
        }
        tmem_wait_st();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[t]);
    }
    if (ok && mbar_wait(&o_full[t], 0, status, 218)) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll 1
      for (int c = 0; c < 128; c += 32) {
        float ov[32];
        tmem_ld32(tO + c, ov);
        tmem_wait_ld();
        if (valid) {
          uint4* dst = reinterpret_cast<uint4*>(O + (int64_t)s * o_ss + h * HD + c);
#pragma unroll
          for (int q = 0; q < 4; ++q)
            dst[q] = make_uint4(pack_bf16x2(ov[8 * q] * inv, ov[8 * q + 1] * inv),
                                pack_bf16x2(ov[8 * q + 2] * inv, ov[8 * q + 3] * inv),
                                pack_bf16x2(ov[8 * q + 4] * inv, ov[8 * q + 5] * inv),
                                pack_bf16x2(ov[8 * q + 6] * inv, ov[8 * q + 7] * inv));
        }
      }
      if (valid) lse[(int64_t)h * g.S + s] = (m + log2f(l)) * kLn2;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

bool attn_tc_eligible(int dtype, int64_t B, int64_t S, int Hq, int Hkv, int hd, int layout,
                      const void* q, int64_t q_ss, const void* k, int64_t k_ss, const void* v,
                      int64_t v_ss) {
  // (tiles of 128 slots index gridDim.y, at most 65535)
  return dtype == PE_BF16 && B == 1 && hd == HD && layout == PE_LAYOUT_PARTITION &&
         S > 0 && S <= 65535ll * TQ && al16(q) && al16(k) && al16(v) && q_ss % 8 == 0 &&
         k_ss % 8 == 0 && v_ss % 8 == 0 && q_ss >= (int64_t)Hq * HD && k_ss >= (int64_t)Hkv * HD &&
         v_ss >= (int64_t)Hkv * HD;
}

int attn_fwd_tc_launch(int64_t S, int Hq, int Hkv, const void* q, int64_t q_ss, const void* k,
                       int64_t k_ss, const void* v, int64_t v_ss, void* o, int64_t o_ss,
                       float* lse, const MaskSpec& m, int* status, cudaStream_t st, int variant) {
  PE_CHECK_ARG(o_ss % 8 == 0 && al16(o), "attention (tcgen05): output must be 16-byte aligned");
  PartGeom g{(int)S, (int)m.a0, (int)m.a1, m.kd - 1};
  if (variant == 1) {
    CUtensorMap tq, tk, tv;
    int rc = make_tmap_2d(&tq, q, (uint64_t)Hq * HD, (uint64_t)S, (uint64_t)q_ss * 2, 64, TQ);
    if (!rc) rc = make_tmap_2d(&tk, k, (uint64_t)Hkv * HD, (uint64_t)S, (uint64_t)k_ss * 2, 64, TK);
    if (!rc) rc = make_tmap_2d(&tv, v, (uint64_t)Hkv * HD, (uint64_t)S, (uint64_t)v_ss * 2, 64, TK);
    if (rc) return rc;
    const float scale_log2 = kLog2e / sqrtf((float)HD);
    PE_CUDA_TRY(cudaFuncSetAttribute(attn_fwd_tc_kernel,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_FWD));
    dim3 grid((unsigned)Hq, (unsigned)((S + TQ - 1) / TQ));
    attn_fwd_tc_kernel<<<grid, kThreads, SMEM_FWD, st>>>(tq, tk, tv, (__nv_bfloat16*)o, o_ss, lse,
                                                         g, Hq, Hq / Hkv, scale_log2, status);
    PE_LAUNCHED();
    return PE_OK;
  }
  return attn_fwd_tc_segments(1, &g, Hq, Hkv, q, q_ss, k, k_ss, v, v_ss, o, o_ss, lse, status, st,
                              -1);
}

int attn_fwd_tc_segments(int nseg, const PartGeom* g, int Hq, int Hkv, const void* q,
                         int64_t q_ss, const void* k, int64_t k_ss, const void* v, int64_t v_ss,
                         void* o, int64_t o_ss, float* lse, int* status, cudaStream_t st,
                         int emu) {
  PE_CHECK_ARG(o_ss % 8 == 0 && al16(o), "attention (tcgen05): output must be 16-byte aligned");
  if (emu < 0) emu = kEmuDefault;
  auto kern = emu == 0 ? attn_fwd_tc2_kernel<0>
              : emu == 2 ? attn_fwd_tc2_kernel<2>
              : emu == 3 ? attn_fwd_tc2_kernel<3>
              : emu == 6 ? attn_fwd_tc2_kernel<6>
              : emu == 8 ? attn_fwd_tc2_kernel<8>
                         : attn_fwd_tc2_kernel<4>;
  PE_CHECK_ARG(emu == 0 || emu == 2 || emu == 3 || emu == 4 || emu == 6 || emu == 8,
               "attention (tcgen05): exp emulation ratio %d not 0/2/3/4/6/8", emu);
  PE_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)SMEM_FWD2));
  {
    // the warpgroups' register re-split assumes the launch grants 168 per thread:
    // with fewer, setmaxnreg.inc would wait for registers that never free up
    cudaFuncAttributes fa;
    PE_CUDA_TRY(cudaFuncGetAttributes(&fa, kern));
    PE_CHECK_ARG(fa.numRegs * kThreads2 >= 4 * 32 * kRegsLow + 8 * 32 * kRegsHigh,
                 "attention (tcgen05): forward kernel compiled with too few registers");
  }
  const float scale_log2 = kLog2e / sqrtf((float)HD);
  // a unit is a pair of query tiles; its cost the key tiles both tiles visit
  auto units = [](const PartGeom& sg) { return (sg.S + 2 * TQ - 1) / (2 * TQ); };
  auto cost = [](const PartGeom& sg, int pr) {
    int c = 0;
    for (int t = 0; t < 2; ++t) {
      const int q0 = (2 * pr + t) * TQ;
      if (q0 >= sg.S) break;
      int r_end, m_beg, m_end;
      key_tiles(sg, q0, r_end, m_beg, m_end, TK);
      c += r_end + (m_end - m_beg);
    }
    return c;
  };
  std::vector<int64_t> rows(nseg + 1, 0);  // first stacked row of every segment
  for (int s = 0; s < nseg; ++s) rows[s + 1] = rows[s] + g[s].S;
  for (auto [b, e] : seg_groups(nseg, g)) {
    SegTable tab;
    memset(&tab, 0, sizeof(tab));
    tab.nseg = e - b;
    int max_units = 0;
    for (int s = b; s < e; ++s) {
      const int i = s - b;
      PE_CHECK_ARG(rows[s] - rows[b] < (1ll << 31), "attention: stacked rows exceed int range");
      tab.g[i] = g[s];
      tab.row0[i] = (int)(rows[s] - rows[b]);
      int rc = seg_map(&tab.tm[i][0], q, rows[s], q_ss, (int64_t)Hq * HD, g[s].S, TQ);
      if (!rc) rc = seg_map(&tab.tm[i][1], k, rows[s], k_ss, (int64_t)Hkv * HD, g[s].S, TK);
      if (!rc) rc = seg_map(&tab.tm[i][2], v, rows[s], v_ss, (int64_t)Hkv * HD, g[s].S, TK);
      if (rc) return rc;
      max_units = std::max(max_units, units(g[s]));
    }
    int rc = seg_table_order(tab, units, cost);
    if (rc) return rc;
    const int ny = tab.nwork > 0 ? tab.nwork : max_units;
    PE_CHECK_ARG(ny <= 65535, "attention: too many query tiles for one launch");
    dim3 grid((unsigned)Hq, (unsigned)ny);
    __nv_bfloat16* ob = static_cast<__nv_bfloat16*>(o) + rows[b] * o_ss;
    kern<<<grid, kThreads2, SMEM_FWD2, st>>>(tab, ob, o_ss, lse + (int64_t)Hq * rows[b], Hq,
                                             Hq / Hkv, scale_log2, status);
    PE_LAUNCHED();
  }
  return PE_OK;
}

}  // namespace pe
