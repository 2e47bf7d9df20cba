// Shared pieces of the tensor-core attention kernels: tile geometry, the
// partition-layout slot decode and the 128-byte shared-memory swizzle.
#pragma once
#include <algorithm>
#include <vector>

#include "attn.cuh"
#include "sm100.cuh"

namespace pe {
namespace attn_tc {

constexpr int HD = 128;  // head dim
constexpr int TQ = 128;  // query rows per tile
constexpr int TK = 128;  // keys per tile
constexpr uint32_t TILE_BYTES = 128 * HD * 2;  // one 128 x 128 bf16 tile = two 64-column chunks
constexpr uint32_t CHUNK = TILE_BYTES / 2;      // 16 KB: 128 rows x 128 B
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// geometry helpers run on the device and, for work-list costs, on the host
#define PE_HD __host__ __device__ __forceinline__
PE_HD int imin(int a, int b) { return a < b ? a : b; }
PE_HD int imax(int a, int b) { return a > b ? a : b; }

// anchor / depth of slot s in the partition layout (reference partition.py:41-55)
PE_HD void decode(const PartGeom& g, int s, int& i, int& d) {
  if (s < g.a1 || g.km1 == 0) {
    i = s;
    d = 0;
  } else {
    const int t = s - g.a1;
    i = g.a0 + t / g.km1;
    d = 1 + t % g.km1;
  }
}

// byte offset of 16-byte unit u (0..7) of row r inside a 128B-swizzled chunk
// (the layout TMA writes with CU_TENSOR_MAP_SWIZZLE_128B on a 1024 B-aligned base)
__device__ __forceinline__ uint32_t swz(int r, int u) {
  return (uint32_t)(r * 128 + ((u ^ (r & 7)) << 4));
}

inline bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---------------------------------------------------- backward tile lists ----
// Up to three disjoint, ascending index ranges [b_i, e_i) (empty ranges are
// b = e = kEmpty and sort last).  Every member is indexed statically, so the
// struct lives in registers.
struct Ranges {
  static constexpr int kEmpty = 0x3fffffff;
  int b0, e0, b1, e1, b2, e2;
  PE_HD int count() const { return (e0 - b0) + (e1 - b1) + (e2 - b2); }
  __device__ __forceinline__ int at(int j) const {
    if (j < e0 - b0) return b0 + j;
    j -= e0 - b0;
    if (j < e1 - b1) return b1 + j;
    return b2 + (j - (e1 - b1));
  }
};

PE_HD void sort2(int& b0, int& e0, int& b1, int& e1) {
  if (b1 < b0) {
    const int tb = b0, te = e0;
    b0 = b1; e0 = e1;
    b1 = tb; e1 = te;
  }
}

// query tiles (of tq rows) whose rows can read some key of key tile [k0, k0 + TK)
PE_HD Ranges query_tiles(const PartGeom& g, int k0, int tq = TQ) {
  constexpr int E = Ranges::kEmpty;
  const int k1 = imin(k0 + TK, g.S);
  const int nqt = (g.S + tq - 1) / tq;
  int b0 = E, e0 = E, b1 = E, e1 = E, b2 = E, e2 = E;
  if (k0 < g.a1) {
    b0 = k0 / tq;  // real rows [k0, a1)
    e0 = (g.a1 - 1) / tq + 1;
    const int af = imax(g.a0, k0);  // prediction rows of anchors >= max(a0, k0)
    if (g.km1 > 0 && af < g.a1) {
      b1 = (g.a1 + (af - g.a0) * g.km1) / tq;
      e1 = nqt;
    }
  }
  if (k1 > g.a1 && g.km1 > 0) {  // the prediction keys' own rows
    const int s0 = imax(k0, g.a1);
    const int i_f = g.a0 + (s0 - g.a1) / g.km1;
    const int i_l = g.a0 + (k1 - 1 - g.a1) / g.km1;
    b2 = (g.a1 + (i_f - g.a0) * g.km1) / tq;
    e2 = (g.a1 + (i_l - g.a0 + 1) * g.km1 - 1) / tq + 1;
  }
  // sort by start, then merge overlapping / touching neighbours
  sort2(b0, e0, b1, e1);
  sort2(b1, e1, b2, e2);
  sort2(b0, e0, b1, e1);
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    if (b1 != E && b1 <= e0) {
      e0 = imax(e0, e1);
      b1 = b2; e1 = e2;
      b2 = e2 = E;
    }
  }
  if (b2 != E && b2 <= e1) {
    e1 = imax(e1, e2);
    b2 = e2 = E;
  }
  Ranges R;
  R.b0 = b0; R.e0 = e0; R.b1 = b1; R.e1 = e1; R.b2 = b2; R.e2 = e2;
  return R;
}

// true when every (query in [q0, q0+tq), key in [k0, k0+TK)) pair is allowed:
// all keys real and no query row's anchor below the last key
__device__ __forceinline__ bool tile_fully_allowed(const PartGeom& g, int q0, int k0,
                                                   int tq = TQ) {
  const int k_last = k0 + TK - 1;
  if (k_last >= g.a1 || q0 + tq > g.S) return false;
  int min_anchor = 1 << 30;
  if (q0 < g.a1) min_anchor = q0;
  if (q0 + tq > g.a1) {
    int i, d;
    decode(g, imax(q0, g.a1), i, d);
    min_anchor = imin(min_anchor, i);
  }
  return min_anchor >= k_last;
}

// key tiles (of tk keys) read by query tile [q0, q0 + TQ): [0, r_end) then [m_beg, m_end)
PE_HD void key_tiles(const PartGeom& g, int q0, int& r_end, int& m_beg, int& m_end,
                     int tk = TK) {
  const int last = imin(q0 + TQ, g.S) - 1;
  int i_last, d_last;
  decode(g, last, i_last, d_last);
  const int i_max = q0 < g.a1 ? imax(i_last, imin(last, g.a1 - 1)) : i_last;
  r_end = i_max / tk + 1;
  m_beg = m_end = 0;
  if (last >= g.a1 && g.km1 > 0) {
    const int first = imax(q0, g.a1);
    int i_first, d_first;
    decode(g, first, i_first, d_first);
    const int lo = g.a1 + (i_first - g.a0) * g.km1;
    const int hi = g.a1 + (i_last - g.a0 + 1) * g.km1;
    int mb = lo / tk, me = (hi - 1) / tk + 1;
    if (mb < r_end) mb = r_end;
    if (me > mb) {
      m_beg = mb;
      m_end = me;
    }
  }
}

__device__ __forceinline__ void atomic_add_row32(float* dst, const float* v, float mul) {
  float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
  for (int t = 0; t < 8; ++t)
    atomicAdd(d4 + t, make_float4(v[4 * t] * mul, v[4 * t + 1] * mul, v[4 * t + 2] * mul,
                                  v[4 * t + 3] * mul));
}

// ------------------------------------------------------ stacked segments ----
// One launch covers every segment of a sequence whose segments are stacked in
// one row space: segment s owns rows [row0_s, row0_s + S_s) of Q / K / V / O /
// dO / dQ / dK / dV, and its lse / delta block [Hq, S_s] starts at element
// Hq * row0_s of the lse / delta buffers.  The work units (segment, tile) run
// segment by segment -- the largest segment first, within a segment the
// heaviest tiles first -- so the operands a segment's units share (its K / V,
// and in the dK / dV kernel its Q / dO of every head) stay in L2 while it runs,
// and the next segment's units start on the SMs the current segment's tail
// leaves idle instead of waiting for a new launch.  Each segment has its own
// tensor maps, so a tile that overhangs a segment reads TMA's zero fill,
// exactly as when the segment is launched alone.
constexpr int kMaxSeg = 8;
constexpr int kMaxWork = 1536;
struct SegTable {
  CUtensorMap tm[kMaxSeg][4];  // per segment: Q, K, V, dO (the forward uses Q, K, V)
  PartGeom g[kMaxSeg];
  int row0[kMaxSeg];
  int nseg;
  int nwork;                   // 0: one segment, units in the kernel's built-in order
  int nsplit;                  // dK / dV kernel: units [0, nsplit) run one item per query
                               // head, later ones one item per KV head (all its query heads)
  uint32_t work[kMaxWork];     // segment << 24 | unit, in execution order
};
constexpr int kWorkSegShift = 24;

__device__ __forceinline__ void unpack_work(uint32_t w, int& seg, int& unit) {
  seg = (int)(w >> kWorkSegShift);
  unit = (int)(w & ((1u << kWorkSegShift) - 1));
}

// Fill the work list of segments [0, nseg) (geometry already in t.g): units(g)
// units per segment, ordered by segment size S descending, then by cost(g, unit)
// descending (ties keep segment, then unit order).  With a single segment the
// list stays empty and the kernel uses its own heaviest-first order.
template <class Units, class Cost>
inline int seg_table_order(SegTable& t, Units units, Cost cost) {
  t.nwork = 0;
  if (t.nseg == 1) return PE_OK;
  struct U { int64_t S, c; uint32_t w; };
  std::vector<U> all;
  for (int s = 0; s < t.nseg; ++s) {
    const int n = units(t.g[s]);
    for (int u = 0; u < n; ++u)
      all.push_back({t.g[s].S, (int64_t)cost(t.g[s], u),
                     ((uint32_t)s << kWorkSegShift) | (uint32_t)u});
  }
  PE_CHECK_ARG((int)all.size() <= kMaxWork, "attention: too many tiles for one launch");
  std::stable_sort(all.begin(), all.end(),
                   [](const U& a, const U& b) { return a.S != b.S ? a.S > b.S : a.c > b.c; });
  for (size_t i = 0; i < all.size(); ++i) t.work[i] = all[i].w;
  t.nwork = (int)all.size();
  return PE_OK;
}

}  // namespace attn_tc

// Launch groups share this unit count: 128-row tiles of a segment (every
// kernel's work units -- query-tile pairs, query tiles, key tiles -- are at most
// that many).
inline int seg_tiles(const attn_tc::PartGeom& g) { return (g.S + attn_tc::TQ - 1) / attn_tc::TQ; }

// Launch groups for stacked segments: runs of consecutive segments that fit one
// SegTable (at most kMaxSeg segments and kMaxWork tiles); a segment with more
// tiles forms a group of its own and runs in the kernel's built-in order.
inline std::vector<std::pair<int, int>> seg_groups(int nseg, const attn_tc::PartGeom* g) {
  std::vector<std::pair<int, int>> out;
  int b = 0, acc = 0;
  for (int s = 0; s < nseg; ++s) {
    const int n = seg_tiles(g[s]);
    if (s > b && (s - b >= attn_tc::kMaxSeg || acc + n > attn_tc::kMaxWork)) {
      out.push_back({b, s});
      b = s;
      acc = 0;
    }
    acc += n;
  }
  if (nseg > b) out.push_back({b, nseg});
  return out;
}

// tensor map over rows [row, row + S) of a bf16 row operand (row stride ss elements)
inline int seg_map(CUtensorMap* map, const void* base, int64_t row, int64_t ss, int64_t cols,
                   int S, uint32_t box_rows) {
  return make_tmap_2d(map, static_cast<const uint8_t*>(base) + row * ss * 2, (uint64_t)cols,
                      (uint64_t)S, (uint64_t)ss * 2, 64, box_rows);
}

// persistent dQ kernel (attn_tc_bwd_q.cu): dq (bf16) = scale * sum dS K per query
// tile, for segments [0, nseg) of one launch group (rows relative to the given
// pointers), units claimed from *work_counter (zeroed beforehand)
int attn_bwd_q2_launch(int nseg, const attn_tc::PartGeom* g, int Hq, int Hkv, const void* q,
                       int64_t q_ss, const void* k, int64_t k_ss, const void* v, int64_t v_ss,
                       const void* dout, int64_t do_ss, const float* lse, const float* delta,
                       void* dq, int64_t dq_ss, const void* rope_cs, int64_t cs_ld,
                       int* work_counter, int* status, cudaStream_t st);
// persistent dK / dV kernel (attn_tc_bwd_kv.cu): accumulates fp32 dK, dV of every
// query head into the KV-head accumulators (zeroed beforehand), items claimed from
// *work_counter (zeroed beforehand); same segment convention
int attn_bwd_kv2_launch(int nseg, const attn_tc::PartGeom* g, int Hq, int Hkv, const void* q,
                        int64_t q_ss, const void* k, int64_t k_ss, const void* v, int64_t v_ss,
                        const void* dout, int64_t do_ss, const float* lse, const float* delta,
                        float* dk_acc, float* dv_acc, int* work_counter, int* status,
                        cudaStream_t st);
}  // namespace pe
