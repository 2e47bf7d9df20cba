// Persistent warp-specialised bf16 GEMM on the 5th-generation tensor cores.
//
//   C[m, n] = alpha * sum_k A(m, k) B(n, k) + beta * Cin[m, n]
//
// Each operand may be K-major (unit stride along k: activations and weights in
// the forward pass) or MN-major (unit stride along m / n: the transposed operands
// of the input- and weight-gradient GEMMs), so the three GEMMs of every
// nn.Linear run without transposing anything in HBM.
//
// CTA tile 128 x BN (BN in 128..256, chosen per shape to avoid a nearly empty
// last wave), K slices of 64 (one 128-byte swizzle
// row of bf16).  Warp 0 issues TMA loads into a STAGES-deep shared-memory ring,
// warp 1 issues tcgen05.mma (128 x BN x 16) into a double-buffered TMEM
// accumulator, warps 2-5 drain the other accumulator (tcgen05.ld) and store to
// HBM, so the epilogue of tile i overlaps the main loop of tile i+1.  The grid
// is one CTA per SM; tiles are walked in L2-sized groups of M-tiles so each
// operand streams from HBM about once.
#include "gemm.cuh"
#include "rope.cuh"
#include "sm100.cuh"

namespace pe {
namespace {

using namespace sm100;

constexpr int BM = 128, BK = 64;
constexpr int kThreads = 192;

// epilogue variants
enum : int {
  EPI_STORE = 0,     // C = alpha * acc + beta * Cin
  EPI_STATS = 1,     // C = round(alpha * acc); stats[row, n_tile] = (max, sum exp(c - max))
  EPI_ROWSCALE = 2,  // C = alpha * acc + rowscale[row] * Cin
  EPI_ROPE = 3,      // C = rotate(round(alpha * acc)) on 128-wide heads below rot_cols
  EPI_SWIGLU = 4,    // gate|up tile pairs: C[:, j], C[:, I + j] = g, u; act[:, j] = silu(g) u
  EPI_SWIGLU_BWD = 5,  // acc = d act[:, j]: C[:, j], C[:, I + j] = d gate, d up (gate|up read)
  EPI_PEXP = 6,        // z = round(alpha * acc); C = e^(z - rowref[row]); stats = (max z, sum C)
};

// EPI_PEXP: the largest amount by which a tile's logits may exceed the row's reference
// (the running maximum of the earlier vocabulary chunks).  e^64 ~ 6e27 keeps every
// exponential, its 128-column sums and the dH accumulation over a chunk finite in fp32
// and bf16; a larger excess sets the overflow word and the caller recomputes the call.
constexpr float kPexpMargin = 64.f;
struct EpiArgs {
  float2* stats;
  int stats_ld;
  const float* rowscale;
  // tile order: 0 automatic; G > 0 groups of G M-tiles (all N-tiles of a group
  // before the next); G < 0 groups of -G N-tiles (all M-tiles of a group first)
  int raster;
  // EPI_ROPE: per-row [cos 64 | sin 64] bf16 table (row stride cs_ld) and the
  // columns [0, rot_cols) whose 128-wide heads are rotated
  const __nv_bfloat16* rope_cs = nullptr;
  int64_t cs_ld = 0;
  int64_t rot_cols = 0;
  // EPI_SWIGLU: intermediate size I (B rows [0, I) gate, [I, 2I) up; a tile of BN
  // columns holds gate rows [tn BN/2, tn BN/2 + BN/2) and the matching up rows) and
  // the activation output
  int64_t swiglu_i = 0;
  __nv_bfloat16* act = nullptr;
  int64_t ld_act = 0;
  // EPI_SWIGLU_BWD: the forward's gate|up rows [M, 2I] (row stride ld_gu); C is the
  // gate|up gradient and the accumulator the activation's gradient
  const __nv_bfloat16* gu = nullptr;
  int64_t ld_gu = 0;
  // plain epilogues: store C with the L2 evict-first policy (C is not read again by
  // this kernel; its lines then leave L2 before the operand panels)
  int store_hint = 0;
  // EPI_PEXP: per-row reference (running maximum), labels (the label column of row r
  // is labels[r] - label_v0; a negative label ignores the row: C = 0), the label
  // logit output and the overflow word (set to 1 when a logit exceeds its row's
  // reference by more than kPexpMargin)
  const float* rowref = nullptr;
  const int64_t* labels = nullptr;
  int64_t label_v0 = 0;
  float* zlab = nullptr;
  int* overflow = nullptr;
  // every variant: when non-null and *run_if == 0 the launch does nothing (every CTA
  // returns before touching its barriers or TMEM) -- a device-side condition for a
  // pass the host enqueues unconditionally
  const int* run_if = nullptr;
};

// silu(g) = g * sigmoid(g) with sigmoid(g) = 1 / (1 + e^-g) from the hardware exp2 and
// reciprocal approximations -- the expression the element-wise SwiGLU kernels use, so
// the fused epilogue gives the same bits -- cheap enough for the epilogue warps
__device__ __forceinline__ float silu_sigmoid(float x) { return __fdividef(1.0f, 1.0f + __expf(-x)); }

// B row of tile column t0 (the first column of a CTA's B sub-tile): the plain
// layout, or for EPI_SWIGLU the gate (t0 < BN/2) or up row it pairs with
template <int BN, int EPI>
__device__ __forceinline__ int b_row_of(int tn, int t0, const EpiArgs& ea) {
  if constexpr (EPI == EPI_SWIGLU) {
    return t0 < BN / 2 ? tn * (BN / 2) + t0 : (int)ea.swiglu_i + tn * (BN / 2) + (t0 - BN / 2);
  } else {
    return tn * BN + t0;
  }
}

constexpr uint32_t pow2_at_least(uint32_t x) {
  uint32_t p = 32;
  while (p < x) p <<= 1;
  return p;
}

template <int BN>
struct TcCfg {
  static_assert(BN % 32 == 0 && BN >= 64 && BN <= 256, "tile width");
  static constexpr uint32_t A_BYTES = BM * BK * 2;
  static constexpr uint32_t B_BYTES = BN * BK * 2;
  static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
  // as many ring stages as fit in ~220 KB of shared memory (at most 8)
  static constexpr int STAGES = (220u * 1024u / STAGE_BYTES) > 8 ? 8 : (220u * 1024u / STAGE_BYTES);
  static constexpr uint32_t TMEM_COLS = pow2_at_least(2 * BN);  // double-buffered accumulator
  static constexpr size_t SMEM = (size_t)STAGES * STAGE_BYTES + 1024 + 256;
};

// Tile width for an M x N problem: the candidate that minimises the predicted
// time ceil(tiles / SMs) * per-tile cost, so a problem of 3.03 waves at 256 wide
// does not pay for a nearly empty fourth wave.  Narrower tiles stream more
// operand bytes per FLOP; the factors below are their relative per-tile speed.
// MN-major B is loaded in 64-column boxes, so its width must be a multiple of 64.
int choose_bn(int64_t M, int64_t N, bool b_mn, int sms) {
  struct Cand {
    int bn;
    float speed;
  };
  static const Cand cands[] = {{256, 1.00f}, {224, 0.97f}, {192, 0.95f}, {160, 0.93f}, {128, 0.88f}};
  const int64_t tm = (M + BM - 1) / BM;
  int best = 256;
  double best_t = 1e30;
  for (const Cand& c : cands) {
    if (b_mn && c.bn % 64 != 0) continue;
    const int64_t tiles = tm * ((N + c.bn - 1) / c.bn);
    const int64_t waves = (tiles + sms - 1) / sms;
    const double t = (double)waves * c.bn / c.speed;
    if (t < best_t - 1e-9) {
      best_t = t;
      best = c.bn;
    }
  }
  return best;
}

// Pair tile width (tiles 256 x BN over the resident clusters): predicted time =
// waves x per-tile cost.  Wider tiles stage fewer operand bytes per FLOP through
// L2 and shared memory, which under the power cap buys clock (the speed factors),
// but tiles wider than 256 use all of TMEM for one accumulator, so their epilogue
// is not hidden behind the next tile's main loop: measured on B200, a 512-wide
// tile's drain costs as much as ~740 K-steps of its main loop with bf16 output
// (twice that with fp32), so wide tiles win only for long K.  MN-major B
// sub-tiles need 64-column boxes.
int choose_bn_pair(int64_t M, int64_t N, int64_t K, bool b_mn, int out_bytes, int clusters) {
  struct Cand {
    int bn;
    float speed;
  };
  static const Cand cands[] = {{512, 1.00f}, {384, 0.97f}, {256, 0.88f}, {192, 0.84f}, {128, 0.78f}};
  const int64_t tm = (M + 2 * BM - 1) / (2 * BM);
  int best = 256;
  double best_t = 1e30;
  for (const Cand& c : cands) {
    const int nj = c.bn > 256 ? c.bn / 2 : c.bn;
    if (b_mn && (nj / 2) % 64 != 0) continue;
    const int64_t tiles = tm * ((N + c.bn - 1) / c.bn);
    const int64_t waves = (tiles + clusters - 1) / clusters;
    const double bubble = c.bn > 256 ? 740.0 * (out_bytes / 2.0) * c.bn / 512.0 : 0.0;
    const double t = (double)waves * c.bn * ((double)K + bubble) / c.speed;
    if (t < best_t - 1e-9) {
      best_t = t;
      best = c.bn;
    }
  }
  return best;
}

// Tiles are walked in groups of G M-tiles (all N-tiles of a group before the next
// group) or, with n_major, groups of G N-tiles: the group's panels of one operand
// stay in L2 while the other operand streams past them.
__device__ __forceinline__ void tile_coords(int tile, int tiles_m, int tiles_n, int G, bool n_major,
                                            int& tm, int& tn) {
  const int outer = n_major ? tiles_n : tiles_m;
  const int inner = n_major ? tiles_m : tiles_n;
  const int per_group = G * inner;
  const int g = tile / per_group;
  const int first = g * G;
  const int gsize = min(outer - first, G);
  const int r = tile - g * per_group;
  const int o = first + r % gsize, i = r / gsize;
  tm = n_major ? i : o;
  tn = n_major ? o : i;
}

// Group size for the tile order: an explicit EpiArgs::raster, else as many M-tiles
// as keep ~40 MB of A panels resident (at least `min_g`).
__device__ __forceinline__ int raster_group(int raster, int tiles_m, int tiles_n, int64_t a_panel,
                                            int min_g, bool& n_major) {
  n_major = raster < 0;
  if (raster != 0) return max(1, min(n_major ? -raster : raster, n_major ? tiles_n : tiles_m));
  return min(tiles_m, max(min_g, (int)((40ll << 20) / a_panel)));
}

template <typename OutT>
__device__ __forceinline__ void store_row32(OutT* dst, const OutT* cin, const float* v, float alpha,
                                            float beta, int valid, bool vec_ok,
                                            const uint64_t* pol = nullptr) {
  float o[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) o[i] = alpha * v[i];
  if (vec_ok && valid == 32) {
    if constexpr (sizeof(OutT) == 2) {
      if (cin) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 u = reinterpret_cast<const uint4*>(cin)[q];
          const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float2 f = __bfloat1622float2(h[j]);
            o[q * 8 + 2 * j] += beta * f.x;
            o[q * 8 + 2 * j + 1] += beta * f.y;
          }
        }
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 u;
        u.x = pack_bf16x2(o[q * 8 + 0], o[q * 8 + 1]);
        u.y = pack_bf16x2(o[q * 8 + 2], o[q * 8 + 3]);
        u.z = pack_bf16x2(o[q * 8 + 4], o[q * 8 + 5]);
        u.w = pack_bf16x2(o[q * 8 + 6], o[q * 8 + 7]);
        if (pol)
          st_v4_hint(reinterpret_cast<uint4*>(dst) + q, u, *pol);
        else
          reinterpret_cast<uint4*>(dst)[q] = u;
      }
    } else {
      if (cin) {
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          float4 f = reinterpret_cast<const float4*>(cin)[q];
          o[4 * q] += beta * f.x;
          o[4 * q + 1] += beta * f.y;
          o[4 * q + 2] += beta * f.z;
          o[4 * q + 3] += beta * f.w;
        }
      }
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 f = make_float4(o[4 * q], o[4 * q + 1], o[4 * q + 2], o[4 * q + 3]);
        if (pol)
          st_v4_hint(reinterpret_cast<float4*>(dst) + q,
                     make_uint4(__float_as_uint(f.x), __float_as_uint(f.y), __float_as_uint(f.z),
                                __float_as_uint(f.w)),
                     *pol);
        else
          reinterpret_cast<float4*>(dst)[q] = f;
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      if (i < valid) {
        float t = o[i];
        if (cin) t += beta * to_f(cin[i]);
        dst[i] = from_f<OutT>(t);
      }
    }
  }
}

// EPI_ROPE drain: columns [c_begin, c_end) are whole 128-wide heads (col0, c_begin,
// c_end and N multiples of 128).  Each head's pair halves (d, d + 64) are read
// together 16 columns at a time, rounded to bf16 as the plain store would round
// them, rotated with the row's table entries when the head lies below rot_cols
// (the q and k heads of a fused q|k|v projection), and stored.
__device__ __forceinline__ void epilogue_rope(uint32_t acc_tmem, int c_begin, int c_end, int64_t gm,
                                              int64_t col0, int M, int N, __nv_bfloat16* C,
                                              int64_t ldc, float alpha, const EpiArgs& ea) {
  const bool row_ok = gm < M;
  const __nv_bfloat16* cs = ea.rope_cs + (row_ok ? gm : 0) * ea.cs_ld;
#pragma unroll 1
  for (int h0 = c_begin; h0 < c_end; h0 += 128) {
    const int64_t gh = col0 + h0;
    const bool rot = gh < ea.rot_cols;
#pragma unroll 1
    for (int jp = 0; jp < 64; jp += 16) {
      float va[16], vb[16];
      tmem_ld16(acc_tmem + h0 + jp, va);
      tmem_ld16(acc_tmem + h0 + 64 + jp, vb);
      tmem_wait_ld();
      if (row_ok && gh < N) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          va[i] = rb16(alpha * va[i]);
          vb[i] = rb16(alpha * vb[i]);
        }
        if (rot) {
          float c[16], sn[16];
          load_bf16_f32<16>(cs + jp, c);
          load_bf16_f32<16>(cs + 64 + jp, sn);
#pragma unroll
          for (int i = 0; i < 16; ++i) rope_rotate_pair(va[i], vb[i], c[i], sn[i], false);
        }
        // each half's 32 bytes as two back-to-back stores: whole sectors after L1 merging
        uint4* da = reinterpret_cast<uint4*>(C + gm * ldc + gh + jp);
#pragma unroll
        for (int q = 0; q < 2; ++q)
          da[q] = make_uint4(pack_bf16x2(va[8 * q], va[8 * q + 1]), pack_bf16x2(va[8 * q + 2], va[8 * q + 3]),
                             pack_bf16x2(va[8 * q + 4], va[8 * q + 5]), pack_bf16x2(va[8 * q + 6], va[8 * q + 7]));
        uint4* db = reinterpret_cast<uint4*>(C + gm * ldc + gh + 64 + jp);
#pragma unroll
        for (int q = 0; q < 2; ++q)
          db[q] = make_uint4(pack_bf16x2(vb[8 * q], vb[8 * q + 1]), pack_bf16x2(vb[8 * q + 2], vb[8 * q + 3]),
                             pack_bf16x2(vb[8 * q + 4], vb[8 * q + 5]), pack_bf16x2(vb[8 * q + 6], vb[8 * q + 7]));
      }
    }
  }
}

// EPI_SWIGLU drain: gate columns [g_begin, g_end) of the tile (TMEM columns from
// acc_tmem) and their up partners half_bn columns on, for intermediate columns
// j0 + c.  g and u are rounded to bf16 as the plain store would round them and
// stored into the gate|up output (the backward reads them); the activation is
// round(round(silu(g)) * u), the element-wise SwiGLU kernels' rounding.
__device__ __forceinline__ void epilogue_swiglu(uint32_t acc_tmem, int g_begin, int g_end,
                                                int half_bn, int64_t gm, int64_t j0, int M,
                                                __nv_bfloat16* C, int64_t ldc, float alpha,
                                                const EpiArgs& ea) {
  const bool row_ok = gm < M;
  const int64_t I = ea.swiglu_i;
  const uint64_t pol = l2_evict_first_policy();
#pragma unroll 1
  for (int c = g_begin; c < g_end; c += 32) {
    float g[32], u[32];
    tmem_ld32(acc_tmem + c, g);
    tmem_ld32(acc_tmem + half_bn + c, u);
    tmem_wait_ld();
    const int64_t j = j0 + c;
    if (row_ok && j < I) {
      // each output's 64 bytes of this row go out as four back-to-back 16-byte stores,
      // so L1 merges them into whole 32-byte sectors (interleaving the three outputs'
      // stores left half-sector writes that L2 must read-modify-write)
      uint32_t pk[16];
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        g[e] = rb16(alpha * g[e]);
        u[e] = rb16(alpha * u[e]);
      }
      uint4* dg = reinterpret_cast<uint4*>(C + gm * ldc + j);
#pragma unroll
      for (int e = 0; e < 16; ++e) pk[e] = pack_bf16x2(g[2 * e], g[2 * e + 1]);
#pragma unroll
      for (int q = 0; q < 4; ++q) st_v4_hint(dg + q, make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]), pol);
      uint4* du = reinterpret_cast<uint4*>(C + gm * ldc + I + j);
#pragma unroll
      for (int e = 0; e < 16; ++e) pk[e] = pack_bf16x2(u[2 * e], u[2 * e + 1]);
#pragma unroll
      for (int q = 0; q < 4; ++q) st_v4_hint(du + q, make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]), pol);
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const float a0 = rb16(g[2 * e] * silu_sigmoid(g[2 * e])) * u[2 * e];
        const float a1 = rb16(g[2 * e + 1] * silu_sigmoid(g[2 * e + 1])) * u[2 * e + 1];
        pk[e] = pack_bf16x2(a0, a1);
      }
      uint4* da = reinterpret_cast<uint4*>(ea.act + gm * ea.ld_act + j);
#pragma unroll
      for (int q = 0; q < 4; ++q) st_v4_hint(da + q, make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]), pol);
    }
  }
}

// EPI_SWIGLU_BWD drain: tile columns [c_begin, c_end) (TMEM columns from acc_tmem) hold
// the activation gradient d of intermediate columns col0 + c.  With g, u the forward's
// gate and up values: d up = d * round(g s), d gate = round(d u) * s (1 + g (1 - s)),
// s = sigmoid(g), d rounded to bf16 first -- the element-wise SwiGLU backward applied
// to the bf16 activation gradient the plain GEMM would store, so both give the same
// bits.  Each thread's 64-byte pieces of g and u are loaded before the accumulator
// columns are read, so the loads overlap the TMEM round trip.
__device__ __forceinline__ void load_bf16x32(const __nv_bfloat16* p, float* f) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint4 w = reinterpret_cast<const uint4*>(p)[q];
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 t = __bfloat1622float2(h[e]);
      f[8 * q + 2 * e] = t.x;
      f[8 * q + 2 * e + 1] = t.y;
    }
  }
}

__device__ __forceinline__ void epilogue_swiglu_bwd(uint32_t acc_tmem, int c_begin, int c_end,
                                                    int64_t gm, int64_t col0, int M,
                                                    __nv_bfloat16* C, int64_t ldc, float alpha,
                                                    const EpiArgs& ea) {
  const bool row_ok = gm < M;
  const int64_t I = ea.swiglu_i;
#pragma unroll 1
  for (int c = c_begin; c < c_end; c += 32) {
    const int64_t j = col0 + c;
    const bool ok = row_ok && j < I;
    float g[32], u[32], d[32];
    if (ok) {
      load_bf16x32(ea.gu + gm * ea.ld_gu + j, g);
      load_bf16x32(ea.gu + gm * ea.ld_gu + I + j, u);
    }
    tmem_ld32(acc_tmem + c, d);
    tmem_wait_ld();
    if (ok) {
      uint32_t pg[16], pu[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        float dg2[2], du2[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int i = 2 * e + h;
          const float dv = rb16(alpha * d[i]);
          const float sg = silu_sigmoid(g[i]);
          const float act = rb16(g[i] * sg);
          const float dact = rb16(dv * u[i]);
          du2[h] = dv * act;
          dg2[h] = dact * (sg * (1.0f + g[i] * (1.0f - sg)));
        }
        pg[e] = pack_bf16x2(dg2[0], dg2[1]);
        pu[e] = pack_bf16x2(du2[0], du2[1]);
      }
      uint4* og = reinterpret_cast<uint4*>(C + gm * ldc + j);
      uint4* ou = reinterpret_cast<uint4*>(C + gm * ldc + I + j);
#pragma unroll
      for (int q = 0; q < 4; ++q) og[q] = make_uint4(pg[4 * q], pg[4 * q + 1], pg[4 * q + 2], pg[4 * q + 3]);
#pragma unroll
      for (int q = 0; q < 4; ++q) ou[q] = make_uint4(pu[4 * q], pu[4 * q + 1], pu[4 * q + 2], pu[4 * q + 3]);
    }
  }
}

// Drains accumulator columns [c_begin, c_end) -- TMEM lanes of this warp, starting
// at TMEM column `acc_tmem` -- into row `gm` of C (tile columns from col0),
// applying the epilogue.  EPI_STATS writes one (max, sum-exp) pair per 128 columns,
// so c_begin and c_end must then be multiples of 128.
template <typename OutT, int EPI>
__device__ __forceinline__ void epilogue_cols(uint32_t acc_tmem, int c_begin, int c_end, int64_t gm,
                                              int64_t col0, int M, int N, OutT* C, int64_t ldc,
                                              const OutT* Cin, int64_t ldcin, float alpha,
                                              float beta, int vec_ok, const EpiArgs& ea) {
  if constexpr (EPI == EPI_ROPE) {
    static_assert(sizeof(OutT) == 2, "the rotary epilogue stores bf16");
    epilogue_rope(acc_tmem, c_begin, c_end, gm, col0, M, N, reinterpret_cast<__nv_bfloat16*>(C),
                  ldc, alpha, ea);
    return;
  }
  // EPI_ROWSCALE: the accumulated input is scaled per row (online-softmax correction)
  const float beta_row = (EPI == EPI_ROWSCALE && gm < M) ? ea.rowscale[gm] : beta;
  float m_run = -INFINITY, s_run = 0.f;  // EPI_STATS: running max / sum-exp of a 128-col chunk
  // EPI_PEXP: the row's reference, label column and whether the row is ignored
  float p_ref = 0.f;
  int64_t lab_col = -1;
  bool p_skip = true;
  if constexpr (EPI == EPI_PEXP) {
    if (gm < M) {
      // without labels (soft targets) no row is ignored and no label logit is taken
      const int64_t lab = ea.labels ? ea.labels[gm] : -1;
      p_ref = ea.rowref[gm];
      p_skip = ea.labels != nullptr && lab < 0;
      lab_col = ea.labels ? lab - ea.label_v0 : -1;
    }
  }
  const uint64_t pol_ef = ea.store_hint ? l2_evict_first_policy() : 0ull;
  const uint64_t* pol = ea.store_hint ? &pol_ef : nullptr;
#pragma unroll 1
  for (int c0 = c_begin; c0 < c_end; c0 += 32) {
    float v[32];
    tmem_ld32(acc_tmem + c0, v);
    tmem_wait_ld();
    const int64_t gn0 = col0 + c0;
    if (gm < M && gn0 < N) {
      const int valid = (N - gn0) < 32 ? (int)(N - gn0) : 32;
      if constexpr (EPI == EPI_STATS) {
        // stats of the values as stored (rounded to the output type)
        float cm = -INFINITY;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          v[i] = round_to<OutT>(alpha * v[i]);
          if (i < valid) cm = fmaxf(cm, v[i]);
        }
        const float mn = fmaxf(m_run, cm);
        float cs = 0.f;
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (i < valid) cs += __expf(v[i] - mn);
        s_run = s_run * __expf(m_run - mn) + cs;
        m_run = mn;
        store_row32<OutT>(C + gm * ldc + gn0, nullptr, v, 1.f, 0.f, valid, vec_ok != 0);
      } else if constexpr (EPI == EPI_PEXP) {
        // the logits as EPI_STATS stores them, then p = e^(z - ref): stats are the
        // tile's maximum logit and its sum of p (relative to ref)
        float cm = -INFINITY, cs = 0.f, zl = 0.f;
        const int64_t lc = lab_col - gn0;
        const bool has_lab = lc >= 0 && lc < valid;
        const int li = has_lab ? (int)lc : -1;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float z = round_to<OutT>(alpha * v[i]);
          cm = i < valid ? fmaxf(cm, z) : cm;
          zl = i == li ? z : zl;
          const float p = p_skip ? 0.f : __expf(z - p_ref);
          cs += i < valid ? p : 0.f;
          v[i] = p;
        }
        if (has_lab) ea.zlab[gm] = zl;
        if (!p_skip && cm - p_ref > kPexpMargin) *ea.overflow = 1;
        m_run = fmaxf(m_run, cm);
        s_run += cs;
        store_row32<OutT>(C + gm * ldc + gn0, nullptr, v, 1.f, 0.f, valid, vec_ok != 0);
      } else {
        store_row32<OutT>(C + gm * ldc + gn0, Cin ? Cin + gm * ldcin + gn0 : nullptr, v, alpha,
                          beta_row, valid, vec_ok != 0, pol);
      }
    }
    if constexpr (EPI == EPI_STATS || EPI == EPI_PEXP) {
      if ((c0 & 127) == 96) {  // end of a 128-column chunk
        const int64_t chunk0 = gn0 - 96;
        if (gm < M && chunk0 < N) ea.stats[gm * ea.stats_ld + chunk0 / 128] = make_float2(m_run, s_run);
        m_run = -INFINITY;
        s_run = 0.f;
      }
    }
  }
}

template <int BN, bool A_MN, bool B_MN, typename OutT, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
               int M, int N, int K, OutT* C, int64_t ldc, const OutT* Cin, int64_t ldcin,
               float alpha, float beta, int vec_ok, EpiArgs ea, int* status) {
  if (ea.run_if != nullptr && *ea.run_if == 0) return;  // a pass the condition skips
  using Cfg = TcCfg<BN>;
  constexpr int STAGES = Cfg::STAGES;
  constexpr uint32_t IDESC = idesc_bf16(BM, BN, A_MN, B_MN);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);
    }
    fence_barrier_init();
    fence_proxy_async();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int tiles_m = (M + BM - 1) / BM;
  const int tiles_n = (N + BN - 1) / BN;
  const int num_tiles = tiles_m * tiles_n;
  const int num_kb = (K + BK - 1) / BK;
  bool n_major;
  const int group_m = raster_group(ea.raster, tiles_m, tiles_n, (int64_t)BM * K * 2, 8, n_major);

  if (warp == 0) {
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int last_stage = -1;
      uint32_t last_phase = 0;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        int tm, tn;
        tile_coords(tile, tiles_m, tiles_n, group_m, n_major, tm, tn);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, status, 101)) { ok = false; break; }
          uint8_t* a_dst = smem + stage * Cfg::STAGE_BYTES;
          uint8_t* b_dst = a_dst + Cfg::A_BYTES;
          mbar_arrive_expect_tx(&full[stage], Cfg::STAGE_BYTES);
          if constexpr (!A_MN) {
            tma_load_2d(a_dst, &tmA, &full[stage], kb * BK, tm * BM);
          } else {
            tma_load_2d(a_dst, &tmA, &full[stage], tm * BM, kb * BK);
            tma_load_2d(a_dst + 8192, &tmA, &full[stage], tm * BM + 64, kb * BK);
          }
          if constexpr (!B_MN) {
            tma_load_2d(b_dst, &tmB, &full[stage], kb * BK, tn * BN);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_2d(b_dst + j * 8192, &tmB, &full[stage], tn * BN + 64 * j, kb * BK);
          }
          last_stage = stage;
          last_phase = phase;
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
      }
      if (!ok && last_stage >= 0) {
        // loads complete in issue order: once the newest one has landed, none of
        // this CTA's copies is still writing shared memory
        mbar_wait(&full[last_stage], last_phase, nullptr, 0);
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1u, status, 102)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, status, 103)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_base = smem_u32(smem + stage * Cfg::STAGE_BYTES);
          const uint32_t b_base = a_base + Cfg::A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = A_MN ? sw128_desc(a_base + k * 2048, 8192, 1024)
                                     : sw128_desc(a_base + k * 32, 16, 1024);
            const uint64_t bd = B_MN ? sw128_desc(b_base + k * 2048, 8192, 1024)
                                     : sw128_desc(b_base + k * 32, 16, 1024);
            mma_bf16_ss(d_tmem, ad, bd, IDESC, (kb | k) != 0 ? 1u : 0u);
          }
          mma_commit(&empty[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
        if (ok) mma_commit(&acc_full[acc]);
      }
    }
  } else {
    // epilogue: warp w reads TMEM lanes 32*(w%4) .. +31
    const int quarter = warp & 3;
    const int row_in_tile = quarter * 32 + lane;
    int local = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      int tm, tn;
      tile_coords(tile, tiles_m, tiles_n, group_m, n_major, tm, tn);
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(&acc_full[acc], acc_phase, status, 104)) break;
      tc_fence_after();
      epilogue_cols<OutT, EPI>(tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN, 0, BN,
                               (int64_t)tm * BM + row_in_tile, (int64_t)tn * BN, M, N, C, ldc, Cin,
                               ldcin, alpha, beta, vec_ok, ea);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[acc]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

// ------------------------------------------------------------------------ //
// CTA-pair variant: a cluster of two CTAs computes a 256 x BN tile with
// tcgen05.mma.cta_group::2.  CTA r of the pair loads A rows [128 r, 128 r + 128)
// and B columns [BN/2 r, BN/2 r + BN/2) of the tile into its own shared memory
// (both loads counted on the leader's `full` barrier), the leader issues the
// MMAs, and each CTA's TMEM receives its 128 accumulator rows.  Per FLOP this
// stages a third fewer operand bytes through L2 and shared memory than the
// single-CTA 128 x 256 tile.
// ------------------------------------------------------------------------ //
constexpr int kPairThreads = 320;  // TMA warp, MMA warp, 8 epilogue warps

template <int BN>
struct PairCfg {
  static_assert(BN % 64 == 0 && BN >= 128 && BN <= 512, "pair tile width");
  static constexpr int NMMA = BN > 256 ? 2 : 1;  // MMAs per K step (N <= 256 each)
  static constexpr int NJ = BN / NMMA;            // N of one MMA
  static constexpr int NJH = NJ / 2;              // B rows of one MMA held by each CTA
  static constexpr int NACC = 2 * BN <= 512 ? 2 : 1;  // TMEM accumulator buffers
  static constexpr uint32_t A_BYTES = BM * BK * 2;
  static constexpr uint32_t BJ_BYTES = NJH * BK * 2;  // one MMA's B sub-tile
  static constexpr uint32_t B_BYTES = NMMA * BJ_BYTES;
  static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (200u * 1024u / STAGE_BYTES) > 8 ? 8 : (200u * 1024u / STAGE_BYTES);
  static constexpr uint32_t TMEM_COLS = NACC == 2 ? pow2_at_least(2 * BN) : 512;
  static constexpr size_t SMEM = (size_t)STAGES * STAGE_BYTES + 1024 + 256;
  static_assert(STAGE_BYTES % 1024 == 0 && BJ_BYTES % 1024 == 0, "1024-byte aligned tiles");
};

template <int BN, bool A_MN, bool B_MN, typename OutT, int EPI>
__global__ void __launch_bounds__(kPairThreads, 1)
gemm_tc_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    int M, int N, int K, OutT* C, int64_t ldc, const OutT* Cin, int64_t ldcin,
                    float alpha, float beta, int vec_ok, EpiArgs ea, int* status) {
  // a pass the condition skips: both CTAs of every pair read the same word and return
  // before any cluster barrier
  if (ea.run_if != nullptr && *ea.run_if == 0) return;
  using Cfg = PairCfg<BN>;
  constexpr int STAGES = Cfg::STAGES;
  constexpr int NMMA = Cfg::NMMA, NJ = Cfg::NJ, NJH = Cfg::NJH, NACC = Cfg::NACC;
  static_assert(!B_MN || NJH % 64 == 0, "MN-major B sub-tiles are loaded in 64-column boxes");
  constexpr uint32_t IDESC = idesc_bf16(2 * BM, NJ, A_MN, B_MN);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* mma_done = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);   // leader: its own arrive + both CTAs' bytes
      mbar_init(&empty[s], 1);  // one MMA commit per consumed stage
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 16);  // 8 epilogue warps in each CTA of the pair
    }
    mbar_init(mma_done, 1);
    fence_barrier_init();
    fence_proxy_async();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish_pair();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers initialised and TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int tiles_m = (M + 2 * BM - 1) / (2 * BM);
  const int tiles_n = (N + BN - 1) / BN;
  const int num_tiles = tiles_m * tiles_n;
  const int num_kb = (K + BK - 1) / BK;
  bool n_major;
  const int group_m =
      raster_group(ea.raster, tiles_m, tiles_n, (int64_t)2 * BM * K * 2, 4, n_major);
  const int cid = (int)cluster_id_x();
  const int ncl = (int)nclusters_x();

  if (warp == 0) {
    if (elect_one()) {
      const uint32_t full_leader = mapa_shared(&full[0], 0);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      bool issued = false;
      for (int tile = cid; tile < num_tiles && ok; tile += ncl) {
        int tm, tn;
        tile_coords(tile, tiles_m, tiles_n, group_m, n_major, tm, tn);
        const int row0 = tm * 2 * BM + (int)rank * BM;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, status, 111)) { ok = false; break; }
          uint8_t* a_dst = smem + stage * Cfg::STAGE_BYTES;
          uint8_t* b_dst = a_dst + Cfg::A_BYTES;
          const uint32_t bar = full_leader + 8u * (uint32_t)stage;
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * Cfg::STAGE_BYTES);
          if constexpr (!A_MN) {
            tma_load_2d_pair(a_dst, &tmA, bar, kb * BK, row0);
          } else {
            tma_load_2d_pair(a_dst, &tmA, bar, row0, kb * BK);
            tma_load_2d_pair(a_dst + 8192, &tmA, bar, row0 + 64, kb * BK);
          }
#pragma unroll
          for (int j = 0; j < NMMA; ++j) {
            // MMA j covers tile columns [j NJ, j NJ + NJ); this CTA holds half of them
            const int bcol0 = b_row_of<BN, EPI>(tn, j * NJ + (int)rank * NJH, ea);
            uint8_t* bj = b_dst + j * Cfg::BJ_BYTES;
            if constexpr (!B_MN) {
              tma_load_2d_pair(bj, &tmB, bar, kb * BK, bcol0);
            } else {
#pragma unroll
              for (int q = 0; q < NJH / 64; ++q)
                tma_load_2d_pair(bj + q * 8192, &tmB, bar, bcol0 + 64 * q, kb * BK);
            }
          }
          issued = true;
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
      }
      if (!ok && issued) {
        // completions are counted on the leader's barrier: give this CTA's copies
        // in flight a bounded moment to land before the CTA can exit
        const uint64_t t0 = globaltimer();
        while (globaltimer() - t0 < 200000ull) {
        }
      }
    }
  } else if (warp == 1) {
    if (leader && elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      bool issued = false;
      for (int tile = cid; tile < num_tiles && ok; tile += ncl, ++local) {
        const int acc = NACC == 2 ? (local & 1) : 0;
        const uint32_t acc_phase = NACC == 2 ? ((local >> 1) & 1) : (local & 1);
        if (!mbar_wait_cluster(&acc_empty[acc], acc_phase ^ 1u, status, 112)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, status, 113)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_base = smem_u32(smem + stage * Cfg::STAGE_BYTES);
          const uint32_t b_base = a_base + Cfg::A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = A_MN ? sw128_desc(a_base + k * 2048, 8192, 1024)
                                     : sw128_desc(a_base + k * 32, 16, 1024);
#pragma unroll
            for (int j = 0; j < NMMA; ++j) {
              const uint32_t bj = b_base + j * Cfg::BJ_BYTES;
              const uint64_t bd = B_MN ? sw128_desc(bj + k * 2048, 8192, 1024)
                                       : sw128_desc(bj + k * 32, 16, 1024);
              mma_bf16_ss_pair(d_tmem + j * NJ, ad, bd, IDESC, (kb | k) != 0 ? 1u : 0u);
            }
          }
          issued = true;
          mma_commit_pair(&empty[stage], 0x3);
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
        if (ok) mma_commit_pair(&acc_full[acc], 0x3);
      }
      if (issued) {
        // every MMA of this pair has finished before TMEM is released
        mma_commit_pair(mma_done, 0x1);
        mbar_wait(mma_done, 0, status, 115);
      }
    }
  } else {
    // epilogue: warp w reads TMEM lanes 32*(w%4) .. +31 of this CTA's 128 rows;
    // warps 2-5 drain the first half of the columns, warps 6-9 the second
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row_in_tile = quarter * 32 + lane;
    const uint32_t acc_empty_leader = mapa_shared(&acc_empty[0], 0);
    int local = 0;
    for (int tile = cid; tile < num_tiles; tile += ncl, ++local) {
      int tm, tn;
      tile_coords(tile, tiles_m, tiles_n, group_m, n_major, tm, tn);
      const int acc = NACC == 2 ? (local & 1) : 0;
      const uint32_t acc_phase = NACC == 2 ? ((local >> 1) & 1) : (local & 1);
      if (!mbar_wait(&acc_full[acc], acc_phase, status, 114)) break;
      tc_fence_after();
      if constexpr (EPI == EPI_SWIGLU) {
        static_assert(sizeof(OutT) == 2 && BN % 64 == 0, "SwiGLU epilogue: bf16, BN % 64 == 0");
        // each warp half drains a quarter of the tile's columns from the gate half and
        // the same quarter from the up half
        epilogue_swiglu(tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN, half * (BN / 4),
                        (half + 1) * (BN / 4), BN / 2,
                        (int64_t)tm * 2 * BM + rank * BM + row_in_tile, (int64_t)tn * (BN / 2), M,
                        reinterpret_cast<__nv_bfloat16*>(C), ldc, alpha, ea);
      } else if constexpr (EPI == EPI_SWIGLU_BWD) {
        static_assert(sizeof(OutT) == 2 && BN % 64 == 0, "SwiGLU backward epilogue: bf16, BN % 64 == 0");
        epilogue_swiglu_bwd(tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN,
                            half * (BN / 2), (half + 1) * (BN / 2),
                            (int64_t)tm * 2 * BM + rank * BM + row_in_tile, (int64_t)tn * BN, M,
                            reinterpret_cast<__nv_bfloat16*>(C), ldc, alpha, ea);
      } else {
        epilogue_cols<OutT, EPI>(tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN,
                                 half * (BN / 2), (half + 1) * (BN / 2),
                                 (int64_t)tm * 2 * BM + rank * BM + row_in_tile, (int64_t)tn * BN,
                                 M, N, C, ldc, Cin, ldcin, alpha, beta, vec_ok, ea);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc_empty_leader + 8u * (uint32_t)acc);
    }
  }

  tc_fence_before();
  cluster_sync();  // neither CTA still touches the other's shared memory or TMEM
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
  }
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

template <int BN, bool A_MN, bool B_MN, typename OutT, int EPI = EPI_STORE>
int launch(const CUtensorMap& ta, const CUtensorMap& tb, int M, int N, int K, void* C, int64_t ldc,
           const void* Cin, int64_t ldcin, float alpha, float beta, int vec_ok, int* status,
           cudaStream_t stream, EpiArgs ea = EpiArgs{}) {
  using Cfg = TcCfg<BN>;
  auto kern = gemm_tc_kernel<BN, A_MN, B_MN, OutT, EPI>;
  PE_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Cfg::SMEM));
  const int tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  const int grid = tiles < sm_count() ? tiles : sm_count();
  kern<<<grid, kThreads, Cfg::SMEM, stream>>>(ta, tb, M, N, K, (OutT*)C, ldc, (const OutT*)Cin,
                                              ldcin, alpha, beta, vec_ok, ea, status);
  PE_LAUNCHED();
  return PE_OK;
}

// Clusters the pair kernel can keep resident at once (one CTA per SM), queried once
// per instantiation; the persistent grid never exceeds it.
template <typename Kern>
int pair_capacity(Kern kern, size_t smem) {
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(2 * (unsigned)(sm_count() / 2), 1, 1);
  cfg.blockDim = dim3(kPairThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
    (void)cudaGetLastError();
    n = sm_count() / 2;
  }
  return n;
}

template <int BN, bool A_MN, bool B_MN, typename OutT, int EPI = EPI_STORE>
int launch_pair(const CUtensorMap& ta, const CUtensorMap& tb, int M, int N, int K, void* C,
                int64_t ldc, const void* Cin, int64_t ldcin, float alpha, float beta, int vec_ok,
                int* status, cudaStream_t stream, EpiArgs ea = EpiArgs{}) {
  using Cfg = PairCfg<BN>;
  auto kern = gemm_tc_pair_kernel<BN, A_MN, B_MN, OutT, EPI>;
  static int capacity[64] = {0};
  int dev = 0;
  PE_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) dev = 0;
  if (capacity[dev] == 0) {
    PE_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Cfg::SMEM));
    capacity[dev] = pair_capacity(kern, Cfg::SMEM);
  }
  const int tiles = ((M + 2 * BM - 1) / (2 * BM)) * ((N + BN - 1) / BN);
  const int clusters = tiles < capacity[dev] ? tiles : capacity[dev];
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(2 * (unsigned)clusters, 1, 1);
  cfg.blockDim = dim3(kPairThreads, 1, 1);
  cfg.dynamicSmemBytes = Cfg::SMEM;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  PE_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, ta, tb, M, N, K, (OutT*)C, ldc, (const OutT*)Cin,
                                 ldcin, alpha, beta, vec_ok, ea, status));
  PE_LAUNCHED();
  return PE_OK;
}

template <int BN, typename OutT>
int launch_majors(bool a_mn, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb, int M, int N,
                  int K, void* C, int64_t ldc, const void* Cin, int64_t ldcin, float alpha,
                  float beta, int vec_ok, int* status, cudaStream_t s, EpiArgs ea) {
  if (!a_mn && !b_mn)
    return launch<BN, false, false, OutT>(ta, tb, M, N, K, C, ldc, Cin, ldcin, alpha, beta, vec_ok, status, s, ea);
  if (!a_mn && b_mn)
    return launch<BN, false, true, OutT>(ta, tb, M, N, K, C, ldc, Cin, ldcin, alpha, beta, vec_ok, status, s, ea);
  if (a_mn && !b_mn)
    return launch<BN, true, false, OutT>(ta, tb, M, N, K, C, ldc, Cin, ldcin, alpha, beta, vec_ok, status, s, ea);
  return launch<BN, true, true, OutT>(ta, tb, M, N, K, C, ldc, Cin, ldcin, alpha, beta, vec_ok, status, s, ea);
}

}  // namespace

bool gemm_tc_eligible(int dtype, int64_t M, int64_t N, int64_t K, const void* A, int64_t a_sm,
                      int64_t a_sk, const void* B, int64_t b_sn, int64_t b_sk, int c_dtype) {
  if (dtype != PE_BF16) return false;
  if (c_dtype != PE_BF16 && c_dtype != PE_F32) return false;
  if (M <= 0 || N <= 0 || K <= 0) return false;
  if (M >= (1ll << 31) || N >= (1ll << 31) || K >= (1ll << 31)) return false;
  if (!al16(A) || !al16(B)) return false;
  // each operand: one unit stride, the other a positive multiple of 8 elements (16 bytes)
  if (a_sk == 1) {
    if (a_sm <= 0 || a_sm % 8 != 0) return false;
  } else if (a_sm == 1) {
    if (a_sk <= 0 || a_sk % 8 != 0) return false;
  } else {
    return false;
  }
  if (b_sk == 1) {
    if (b_sn <= 0 || b_sn % 8 != 0) return false;
  } else if (b_sn == 1) {
    if (b_sk <= 0 || b_sk % 8 != 0) return false;
  } else {
    return false;
  }
  return true;
}

template <int BN, typename OutT>
int launch_bn(bool a_mn, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb, int M, int N,
              int K, void* C, int64_t ldc, const void* Cin, int64_t ldcin, float alpha,
              float beta, int vec_ok, int* status, cudaStream_t s, EpiArgs ea) {
  if constexpr (BN % 64 == 0) {
    return launch_majors<BN, OutT>(a_mn, b_mn, ta, tb, M, N, K, C, ldc, Cin, ldcin, alpha, beta,
                                   vec_ok, status, s, ea);
  } else {
    if (b_mn) {
      set_error("gemm: tile width %d needs a K-major B operand", BN);
      return PE_ERR_ARG;
    }
    if (a_mn)
      return launch<BN, true, false, OutT>(ta, tb, M, N, K, C, ldc, Cin, ldcin, alpha, beta,
                                           vec_ok, status, s, ea);
    return launch<BN, false, false, OutT>(ta, tb, M, N, K, C, ldc, Cin, ldcin, alpha, beta, vec_ok,
                                          status, s, ea);
  }
}

template <typename OutT>
int launch_any_bn(int BN, bool a_mn, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb,
                  int M, int N, int K, void* C, int64_t ldc, const void* Cin, int64_t ldcin,
                  float alpha, float beta, int vec_ok, int* status, cudaStream_t s, EpiArgs ea) {
  switch (BN) {
    case 256: return launch_bn<256, OutT>(a_mn, b_mn, ta, tb, M, N, K, C, ldc, Cin, ldcin, alpha, beta, vec_ok, status, s, ea);
    case 224: return launch_bn<224, OutT>(a_mn, b_mn, ta, tb, M, N, K, C, ldc, Cin, ldcin, alpha, beta, vec_ok, status, s, ea);
    case 192: return launch_bn<192, OutT>(a_mn, b_mn, ta, tb, M, N, K, C, ldc, Cin, ldcin, alpha, beta, vec_ok, status, s, ea);
    case 160: return launch_bn<160, OutT>(a_mn, b_mn, ta, tb, M, N, K, C, ldc, Cin, ldcin, alpha, beta, vec_ok, status, s, ea);
    case 128: return launch_bn<128, OutT>(a_mn, b_mn, ta, tb, M, N, K, C, ldc, Cin, ldcin, alpha, beta, vec_ok, status, s, ea);
    default: break;
  }
  set_error("gemm: unsupported tile width %d", BN);
  return PE_ERR_ARG;
}

template <int BN, typename OutT>
int launch_pair_majors(bool a_mn, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb, int M,
                       int N, int K, void* C, int64_t ldc, const void* Cin, int64_t ldcin,
                       float alpha, float beta, int vec_ok, int* status, cudaStream_t s, EpiArgs ea) {
  if constexpr (PairCfg<BN>::NJH % 64 == 0) {
    if (b_mn) {
      if (a_mn)
        return launch_pair<BN, true, true, OutT>(ta, tb, M, N, K, C, ldc, Cin, ldcin, alpha, beta,
                                                 vec_ok, status, s, ea);
      return launch_pair<BN, false, true, OutT>(ta, tb, M, N, K, C, ldc, Cin, ldcin, alpha, beta,
                                                vec_ok, status, s, ea);
    }
  } else {
    if (b_mn) {
      set_error("gemm: pair tile width %d needs a K-major B operand", BN);
      return PE_ERR_ARG;
    }
  }
  if (a_mn)
    return launch_pair<BN, true, false, OutT>(ta, tb, M, N, K, C, ldc, Cin, ldcin, alpha, beta,
                                              vec_ok, status, s, ea);
  return launch_pair<BN, false, false, OutT>(ta, tb, M, N, K, C, ldc, Cin, ldcin, alpha, beta,
                                             vec_ok, status, s, ea);
}

template <typename OutT>
int launch_pair_any_bn(int BN, bool a_mn, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb,
                       int M, int N, int K, void* C, int64_t ldc, const void* Cin, int64_t ldcin,
                       float alpha, float beta, int vec_ok, int* status, cudaStream_t s, EpiArgs ea) {
  switch (BN) {
    case 512: return launch_pair_majors<512, OutT>(a_mn, b_mn, ta, tb, M, N, K, C, ldc, Cin, ldcin, alpha, beta, vec_ok, status, s, ea);
    case 384: return launch_pair_majors<384, OutT>(a_mn, b_mn, ta, tb, M, N, K, C, ldc, Cin, ldcin, alpha, beta, vec_ok, status, s, ea);
    case 256: return launch_pair_majors<256, OutT>(a_mn, b_mn, ta, tb, M, N, K, C, ldc, Cin, ldcin, alpha, beta, vec_ok, status, s, ea);
    case 192: return launch_pair_majors<192, OutT>(a_mn, b_mn, ta, tb, M, N, K, C, ldc, Cin, ldcin, alpha, beta, vec_ok, status, s, ea);
    case 128: return launch_pair_majors<128, OutT>(a_mn, b_mn, ta, tb, M, N, K, C, ldc, Cin, ldcin, alpha, beta, vec_ok, status, s, ea);
    default: break;
  }
  set_error("gemm: unsupported pair tile width %d", BN);
  return PE_ERR_ARG;
}

// B rows of one MMA held by each CTA of the pair (the TMA box height for K-major B)
int pair_b_box(int bn) { return (bn > 256 ? bn / 2 : bn) / 2; }

// The CTA-pair kernel takes problems with at least this many rows (below it half
// of a 256-row pair tile would mostly be padding).
constexpr int64_t kPairMinRows = 512;

bool use_pair(int64_t M, int mode) {
  if (mode == 1) return false;
  if (mode == 2) return true;
  return M >= kPairMinRows;
}

int gemm_tc(int64_t M, int64_t N, int64_t K, const void* A, int64_t a_sm, int64_t a_sk,
            const void* B, int64_t b_sn, int64_t b_sk, void* C, int64_t ldc, int c_dtype,
            const void* Cin, int64_t ldcin, float alpha, float beta, int* status,
            cudaStream_t stream, int force_bn, int mode, int raster, int store_hint) {
  const bool a_mn = a_sk != 1;
  const bool b_mn = b_sk != 1;
  const bool pair = use_pair(M, mode);
  int BN;
  if (pair) {
    BN = force_bn > 0 ? force_bn
                      : choose_bn_pair(M, N, K, b_mn, c_dtype == PE_F32 ? 4 : 2, sm_count() / 2);
    PE_CHECK_ARG(BN == 128 || BN == 192 || BN == 256 || BN == 384 || BN == 512,
                 "gemm: pair tile width %d not 128/192/256/384/512", BN);
    PE_CHECK_ARG(!(b_mn && pair_b_box(BN) % 64 != 0), "gemm: pair tile width %d needs a K-major B",
                 BN);
  } else {
    BN = force_bn > 0 ? force_bn : choose_bn(M, N, b_mn, sm_count());
    PE_CHECK_ARG(!(b_mn && BN % 64 != 0), "gemm: tile width %d needs a K-major B operand", BN);
  }
  const uint32_t b_box = pair ? (uint32_t)pair_b_box(BN) : (uint32_t)BN;
  CUtensorMap ta, tb;
  int rc;
  if (!a_mn)
    rc = make_tmap_2d(&ta, A, (uint64_t)K, (uint64_t)M, (uint64_t)a_sm * 2, 64, 128);
  else
    rc = make_tmap_2d(&ta, A, (uint64_t)M, (uint64_t)K, (uint64_t)a_sk * 2, 64, 64);
  if (rc) return rc;
  if (!b_mn)
    rc = make_tmap_2d(&tb, B, (uint64_t)K, (uint64_t)N, (uint64_t)b_sn * 2, 64, b_box);
  else
    rc = make_tmap_2d(&tb, B, (uint64_t)N, (uint64_t)K, (uint64_t)b_sk * 2, 64, 64);
  if (rc) return rc;
  const size_t esz = c_dtype == PE_F32 ? 4 : 2;
  const int vec_ok = (ldc * esz) % 16 == 0 && al16(C) &&
                     (!Cin || ((ldcin * esz) % 16 == 0 && al16(Cin)));
  const int m = (int)M, n = (int)N, k = (int)K;
  EpiArgs ea{nullptr, 0, nullptr, raster};
  ea.store_hint = store_hint;
  if (pair) {
    if (c_dtype == PE_F32)
      return launch_pair_any_bn<float>(BN, a_mn, b_mn, ta, tb, m, n, k, C, ldc, Cin, ldcin, alpha,
                                       beta, vec_ok, status, stream, ea);
    return launch_pair_any_bn<__nv_bfloat16>(BN, a_mn, b_mn, ta, tb, m, n, k, C, ldc, Cin, ldcin,
                                             alpha, beta, vec_ok, status, stream, ea);
  }
  if (c_dtype == PE_F32)
    return launch_any_bn<float>(BN, a_mn, b_mn, ta, tb, m, n, k, C, ldc, Cin, ldcin, alpha, beta,
                                vec_ok, status, stream, ea);
  return launch_any_bn<__nv_bfloat16>(BN, a_mn, b_mn, ta, tb, m, n, k, C, ldc, Cin, ldcin, alpha,
                                      beta, vec_ok, status, stream, ea);
}

int gemm_tc_logits_stats(int64_t M, int64_t N, int64_t K, const void* A, int64_t lda,
                         const void* B, int64_t ldb, void* C, int64_t ldc, float2* stats,
                         int stats_ld, int* status, cudaStream_t stream, int force_bn,
                         const int* run_if) {
  PE_CHECK_ARG(M > 0 && N > 0 && K > 0 && lda % 8 == 0 && ldb % 8 == 0 && ldc % 8 == 0 &&
                   al16(A) && al16(B) && al16(C),
               "gemm (logits + row stats): operands must be 16-byte aligned bf16");
  PE_CHECK_ARG(stats_ld >= (N + 127) / 128, "gemm (logits + row stats): stats_ld too small");
  PE_CHECK_ARG(force_bn == 0 || force_bn == 256 || force_bn == 512,
               "gemm (logits + row stats): tile width %d not 256 or 512", force_bn);
  const bool pair = use_pair(M, 0);
  // pair tiles 256 x 512 or 256 x 256 (the stats need 128-column aligned halves)
  const int pbn = !pair ? 256
                  : force_bn ? force_bn
                  : (choose_bn_pair(M, N, K, false, 2, sm_count() / 2) > 256 ? 512 : 256);
  CUtensorMap ta, tb;
  int rc = make_tmap_2d(&ta, A, (uint64_t)K, (uint64_t)M, (uint64_t)lda * 2, 64, 128);
  if (!rc)
    rc = make_tmap_2d(&tb, B, (uint64_t)K, (uint64_t)N, (uint64_t)ldb * 2, 64,
                      pair ? (uint32_t)pair_b_box(pbn) : 256u);
  if (rc) return rc;
  EpiArgs ea{stats, stats_ld, nullptr, 0};
  ea.run_if = run_if;
  if (pair && pbn == 512)
    return launch_pair<512, false, false, __nv_bfloat16, EPI_STATS>(
        ta, tb, (int)M, (int)N, (int)K, C, ldc, nullptr, 0, 1.f, 0.f, 1, status, stream, ea);
  if (pair)
    return launch_pair<256, false, false, __nv_bfloat16, EPI_STATS>(
        ta, tb, (int)M, (int)N, (int)K, C, ldc, nullptr, 0, 1.f, 0.f, 1, status, stream, ea);
  return launch<256, false, false, __nv_bfloat16, EPI_STATS>(ta, tb, (int)M, (int)N, (int)K, C, ldc,
                                                             nullptr, 0, 1.f, 0.f, 1, status,
                                                             stream, ea);
}

// P = e^(round(h W^T) - rowref[row]) (bf16; 0 for rows with a negative label), the
// per-128-column (max logit, sum P) pairs, the label logit of the rows whose label
// falls in these N columns (labels[r] - label_v0; labels may be null: soft targets),
// and *overflow = 1 when a logit exceeds its row's reference by more than
// kPexpMargin.  Tiles as the logits + stats GEMM.
int gemm_tc_logits_pexp(int64_t M, int64_t N, int64_t K, const void* A, int64_t lda,
                        const void* B, int64_t ldb, void* P, int64_t ldp, float2* stats,
                        int stats_ld, const float* rowref, const int64_t* labels,
                        int64_t label_v0, float* zlab, int* overflow, int* status,
                        cudaStream_t stream, int force_bn) {
  PE_CHECK_ARG(M > 0 && N > 0 && K > 0 && lda % 8 == 0 && ldb % 8 == 0 && ldp % 8 == 0 &&
                   al16(A) && al16(B) && al16(P),
               "gemm (logits -> exponentials): operands must be 16-byte aligned bf16");
  PE_CHECK_ARG(stats_ld >= (N + 127) / 128, "gemm (logits -> exponentials): stats_ld too small");
  PE_CHECK_ARG(rowref && overflow && (labels == nullptr || zlab != nullptr),
               "gemm (logits -> exponentials): the reference, the overflow word and, with "
               "labels, the label-logit output are required");
  PE_CHECK_ARG(force_bn == 0 || force_bn == 256 || force_bn == 512,
               "gemm (logits -> exponentials): tile width %d not 256 or 512", force_bn);
  const bool pair = use_pair(M, 0);
  const int pbn = !pair ? 256
                  : force_bn ? force_bn
                  : (choose_bn_pair(M, N, K, false, 2, sm_count() / 2) > 256 ? 512 : 256);
  CUtensorMap ta, tb;
  int rc = make_tmap_2d(&ta, A, (uint64_t)K, (uint64_t)M, (uint64_t)lda * 2, 64, 128);
  if (!rc)
    rc = make_tmap_2d(&tb, B, (uint64_t)K, (uint64_t)N, (uint64_t)ldb * 2, 64,
                      pair ? (uint32_t)pair_b_box(pbn) : 256u);
  if (rc) return rc;
  EpiArgs ea{stats, stats_ld, nullptr, 0};
  ea.rowref = rowref;
  ea.labels = labels;
  ea.label_v0 = label_v0;
  ea.zlab = zlab;
  ea.overflow = overflow;
  if (pair && pbn == 512)
    return launch_pair<512, false, false, __nv_bfloat16, EPI_PEXP>(
        ta, tb, (int)M, (int)N, (int)K, P, ldp, nullptr, 0, 1.f, 0.f, 1, status, stream, ea);
  if (pair)
    return launch_pair<256, false, false, __nv_bfloat16, EPI_PEXP>(
        ta, tb, (int)M, (int)N, (int)K, P, ldp, nullptr, 0, 1.f, 0.f, 1, status, stream, ea);
  return launch<256, false, false, __nv_bfloat16, EPI_PEXP>(ta, tb, (int)M, (int)N, (int)K, P, ldp,
                                                            nullptr, 0, 1.f, 0.f, 1, status,
                                                            stream, ea);
}

int gemm_tc_rowscale_acc(int64_t M, int64_t N, int64_t K, const void* A, int64_t lda,
                         const void* B, int64_t b_sk, float* C, int64_t ldc, const float* Cin,
                         const float* rowscale, int* status, cudaStream_t stream,
                         int force_bn, const int* run_if) {
  PE_CHECK_ARG(M > 0 && N > 0 && K > 0 && lda % 8 == 0 && b_sk % 8 == 0 && ldc % 4 == 0 &&
                   al16(A) && al16(B) && al16(C),
               "gemm (row-scaled accumulate): operands must be 16-byte aligned");
  CUtensorMap ta, tb;
  int rc = make_tmap_2d(&ta, A, (uint64_t)K, (uint64_t)M, (uint64_t)lda * 2, 64, 128);
  if (!rc) rc = make_tmap_2d(&tb, B, (uint64_t)N, (uint64_t)K, (uint64_t)b_sk * 2, 64, 64);
  if (rc) return rc;
  EpiArgs ea{nullptr, 0, rowscale, 0};
  ea.run_if = run_if;
  PE_CHECK_ARG(force_bn == 0 || force_bn == 256 || force_bn == 512,
               "gemm (row-scaled accumulate): tile width %d not 256 or 512", force_bn);
  if (use_pair(M, 0)) {
    const int bn = force_bn ? force_bn : choose_bn_pair(M, N, K, true, 4, sm_count() / 2);
    if (bn == 512)
      return launch_pair<512, false, true, float, EPI_ROWSCALE>(
          ta, tb, (int)M, (int)N, (int)K, C, ldc, Cin, ldc, 1.f, 0.f, 1, status, stream, ea);
    return launch_pair<256, false, true, float, EPI_ROWSCALE>(
        ta, tb, (int)M, (int)N, (int)K, C, ldc, Cin, ldc, 1.f, 0.f, 1, status, stream, ea);
  }
  return launch<256, false, true, float, EPI_ROWSCALE>(ta, tb, (int)M, (int)N, (int)K, C, ldc, Cin,
                                                       ldc, 1.f, 0.f, 1, status, stream, ea);
}

// y = x w^T (bf16, both K-major) with the rotary embedding applied to the 128-wide
// heads of columns [0, rot_cols) in the epilogue.  Tiles are 256 or 512 columns
// wide (CTA pairs) or 256 (single CTAs), so every epilogue warp's column range is
// made of whole heads.
int gemm_tc_rope(int64_t M, int64_t N, int64_t K, const void* A, int64_t lda, const void* B,
                 int64_t ldb, void* C, int64_t ldc, const void* cs, int64_t cs_ld,
                 int64_t rot_cols, int* status, cudaStream_t stream) {
  PE_CHECK_ARG(M > 0 && N > 0 && K > 0, "linear + rope: empty problem");
  PE_CHECK_ARG(N % 128 == 0 && rot_cols % 128 == 0 && rot_cols >= 0 && rot_cols <= N,
               "linear + rope: N and rot_cols must be multiples of head_dim 128 (rot_cols <= N)");
  PE_CHECK_ARG(M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31),
               "linear + rope: dimensions too large");
  PE_CHECK_ARG(lda % 8 == 0 && ldb % 8 == 0 && ldc % 8 == 0 && cs_ld % 8 == 0 && cs_ld >= 128 &&
                   al16(A) && al16(B) && al16(C) && al16(cs),
               "linear + rope: operands and the table must be 16-byte aligned bf16");
  const bool pair = use_pair(M, 0);
  const int pbn = pair ? (choose_bn_pair(M, N, K, false, 2, sm_count() / 2) > 256 ? 512 : 256) : 256;
  CUtensorMap ta, tb;
  int rc = make_tmap_2d(&ta, A, (uint64_t)K, (uint64_t)M, (uint64_t)lda * 2, 64, 128);
  if (!rc)
    rc = make_tmap_2d(&tb, B, (uint64_t)K, (uint64_t)N, (uint64_t)ldb * 2, 64,
                      pair ? (uint32_t)pair_b_box(pbn) : 256u);
  if (rc) return rc;
  EpiArgs ea{nullptr, 0, nullptr, 0};
  ea.rope_cs = static_cast<const __nv_bfloat16*>(cs);
  ea.cs_ld = cs_ld;
  ea.rot_cols = rot_cols;
  if (pair && pbn == 512)
    return launch_pair<512, false, false, __nv_bfloat16, EPI_ROPE>(
        ta, tb, (int)M, (int)N, (int)K, C, ldc, nullptr, 0, 1.f, 0.f, 1, status, stream, ea);
  if (pair)
    return launch_pair<256, false, false, __nv_bfloat16, EPI_ROPE>(
        ta, tb, (int)M, (int)N, (int)K, C, ldc, nullptr, 0, 1.f, 0.f, 1, status, stream, ea);
  return launch<256, false, false, __nv_bfloat16, EPI_ROPE>(ta, tb, (int)M, (int)N, (int)K, C, ldc,
                                                            nullptr, 0, 1.f, 0.f, 1, status,
                                                            stream, ea);
}

// gu = x w_gu^T and act = silu(gate) * up.  On the tensor-core path with CTA-pair
// tiles (M >= 512, bf16, I a multiple of BN/2 for the chosen 256- or 512-wide tile,
// 16-byte aligned rows) the activation is the GEMM epilogue's; otherwise the plain
// GEMM runs, then the element-wise SwiGLU kernel (same bits either way).  algo bits
// 8-17 may force the pair tile width (256 or 512).
int gemm_tc_swiglu(int dtype, int64_t M, int64_t I, int64_t K, const void* A, int64_t lda,
                   const void* B, int64_t ldb, void* C, int64_t ldc, void* act, int64_t ld_act,
                   int algo, int* status, cudaStream_t stream) {
  const int force_bn = (algo >> 8) & 0x3ff;
  PE_CHECK_ARG(force_bn == 0 || force_bn == 256 || force_bn == 512,
               "linear + swiglu: forced tile width %d not 256 or 512", force_bn);
  const int64_t N = 2 * I;
  int pbn = 0;
  bool fused = dtype == PE_BF16 && use_pair(M, 0) && M < (1ll << 31) && N < (1ll << 31) &&
               K < (1ll << 31) && lda % 8 == 0 && ldb % 8 == 0 && ldc % 8 == 0 &&
               ld_act % 8 == 0 && al16(A) && al16(B) && al16(C) && al16(act);
  if (fused) {
    pbn = force_bn ? force_bn
                   : (choose_bn_pair(M, N, K, false, 2, sm_count() / 2) > 256 ? 512 : 256);
    fused = I % (pbn / 2) == 0;
  }
  if (!fused) {
    int rc = gemm(dtype, M, N, K, A, lda, 1, B, ldb, 1, C, ldc, dtype, nullptr, 0, 1.f, 0.f,
                  algo & 0xff, status, stream);
    if (rc) return rc;
    return ::pe_swiglu_fwd(dtype, M, I, C, ldc, act, ld_act, stream);
  }
  CUtensorMap ta, tb;
  int rc = make_tmap_2d(&ta, A, (uint64_t)K, (uint64_t)M, (uint64_t)lda * 2, 64, 128);
  if (!rc)
    rc = make_tmap_2d(&tb, B, (uint64_t)K, (uint64_t)N, (uint64_t)ldb * 2, 64,
                      (uint32_t)pair_b_box(pbn));
  if (rc) return rc;
  EpiArgs ea{nullptr, 0, nullptr, 0};
  ea.swiglu_i = I;
  ea.act = static_cast<__nv_bfloat16*>(act);
  ea.ld_act = ld_act;
  if (pbn == 512)
    return launch_pair<512, false, false, __nv_bfloat16, EPI_SWIGLU>(
        ta, tb, (int)M, (int)N, (int)K, C, ldc, nullptr, 0, 1.f, 0.f, 1, status, stream, ea);
  return launch_pair<256, false, false, __nv_bfloat16, EPI_SWIGLU>(
      ta, tb, (int)M, (int)N, (int)K, C, ldc, nullptr, 0, 1.f, 0.f, 1, status, stream, ea);
}

// dgu = swiglu_backward(dy w, gu): the down projection's input gradient d act = dy w
// (dy [M, K], w [K, I] with row stride ldw) with the SwiGLU backward in the epilogue of
// the CTA-pair GEMM (bf16, M >= 512 rows, I % 32 == 0, 16-byte aligned rows); the
// activation gradient itself is never stored.  Otherwise the plain GEMM writes d act
// into the up half of dgu and the element-wise SwiGLU backward rewrites dgu in place
// (each element's d act is read before its d up is written, by the same thread): the
// same bits either way.  algo bits 8-17 may force the pair tile width (256 or 512).
int gemm_tc_swiglu_bwd(int dtype, int64_t M, int64_t I, int64_t K, const void* dy, int64_t lddy,
                       const void* w, int64_t ldw, const void* gu, int64_t ldgu, void* dgu,
                       int64_t lddgu, int algo, int* status, cudaStream_t stream) {
  const int force_bn = (algo >> 8) & 0x3ff;
  PE_CHECK_ARG(force_bn == 0 || force_bn == 256 || force_bn == 512,
               "linear + swiglu backward: forced tile width %d not 256 or 512", force_bn);
  const bool fused = dtype == PE_BF16 && use_pair(M, 0) && M < (1ll << 31) && I < (1ll << 31) &&
                     K < (1ll << 31) && I % 32 == 0 && lddy % 8 == 0 && ldw % 8 == 0 &&
                     ldgu % 8 == 0 && lddgu % 8 == 0 && al16(dy) && al16(w) && al16(gu) &&
                     al16(dgu);
  if (!fused) {
    const size_t esz = dtype == PE_F32 ? 4 : 2;
    void* da = static_cast<uint8_t*>(dgu) + (size_t)I * esz;
    int rc = gemm(dtype, M, I, K, dy, lddy, 1, w, 1, ldw, da, lddgu, dtype, nullptr, 0, 1.f, 0.f,
                  algo & 0xff, status, stream);
    if (rc) return rc;
    return ::pe_swiglu_bwd(dtype, M, I, da, lddgu, gu, ldgu, dgu, lddgu, stream);
  }
  // 256-wide tiles keep two accumulators in TMEM, so a tile's epilogue (which reads
  // gate|up and writes both gradient halves) runs behind the next tile's main loop
  const int pbn = force_bn ? force_bn : 256;
  CUtensorMap ta, tb;
  int rc = make_tmap_2d(&ta, dy, (uint64_t)K, (uint64_t)M, (uint64_t)lddy * 2, 64, 128);
  if (!rc) rc = make_tmap_2d(&tb, w, (uint64_t)I, (uint64_t)K, (uint64_t)ldw * 2, 64, 64);
  if (rc) return rc;
  EpiArgs ea{nullptr, 0, nullptr, 0};
  ea.swiglu_i = I;
  ea.gu = static_cast<const __nv_bfloat16*>(gu);
  ea.ld_gu = ldgu;
  if (pbn == 512)
    return launch_pair<512, false, true, __nv_bfloat16, EPI_SWIGLU_BWD>(
        ta, tb, (int)M, (int)I, (int)K, dgu, lddgu, nullptr, 0, 1.f, 0.f, 1, status, stream, ea);
  return launch_pair<256, false, true, __nv_bfloat16, EPI_SWIGLU_BWD>(
      ta, tb, (int)M, (int)I, (int)K, dgu, lddgu, nullptr, 0, 1.f, 0.f, 1, status, stream, ea);
}

int gemm(int dtype, int64_t M, int64_t N, int64_t K, const void* A, int64_t a_sm, int64_t a_sk,
         const void* B, int64_t b_sn, int64_t b_sk, void* C, int64_t ldc, int c_dtype,
         const void* Cin, int64_t ldcin, float alpha, float beta, int algo, int* status,
         cudaStream_t stream) {
  PE_CHECK_ARG(M >= 0 && N >= 0 && K >= 0, "gemm: negative size");
  PE_CHECK_ARG(ldc >= N, "gemm: ldc < N");
  if (M == 0 || N == 0) return PE_OK;
  PE_CHECK_ARG(K > 0, "gemm: K == 0 is not supported");
  const int algo_bits = algo;
  const int force_bn = (algo >> 8) & 0x3ff;
  const int mode = (algo >> 20) & 3;  // 0 automatic, 1 single-CTA tiles, 2 CTA-pair tiles
  algo &= 0xff;
  PE_CHECK_ARG(force_bn == 0 || force_bn == 128 || force_bn == 160 || force_bn == 192 ||
                   force_bn == 224 || force_bn == 256 || force_bn == 384 || force_bn == 512,
               "gemm: forced tile width %d not one of 128/160/192/224/256/384/512", force_bn);
  PE_CHECK_ARG(mode != 3, "gemm: tile mode 3 is not defined");
  // bits 24-29: tile-group size (0 automatic); bit 30: group along N instead of M
  const int group = (algo_bits >> 24) & 0x3f;
  const int raster = ((algo_bits >> 30) & 1) ? -group : group;
  // bit 22: store C with the L2 evict-first policy
  const int store_hint = (algo_bits >> 22) & 1;
  const bool tc_ok = gemm_tc_eligible(dtype, M, N, K, A, a_sm, a_sk, B, b_sn, b_sk, c_dtype);
  if (algo == PE_ALGO_TCGEN05) {
    PE_CHECK_ARG(tc_ok, "gemm: operands not eligible for the tcgen05 path");
    return gemm_tc(M, N, K, A, a_sm, a_sk, B, b_sn, b_sk, C, ldc, c_dtype, Cin, ldcin, alpha,
                   beta, status, stream, force_bn, mode, raster, store_hint);
  }
  if (algo == PE_ALGO_AUTO && tc_ok)
    return gemm_tc(M, N, K, A, a_sm, a_sk, B, b_sn, b_sk, C, ldc, c_dtype, Cin, ldcin, alpha,
                   beta, status, stream, force_bn, mode, raster, store_hint);
  return gemm_simt(dtype, M, N, K, A, a_sm, a_sk, B, b_sn, b_sk, C, ldc, c_dtype, Cin, ldcin,
                   alpha, beta, stream);
}

}  // namespace pe

extern "C" int pe_linear_rope(int dtype, int64_t M, int64_t N, int64_t K, const void* x,
                              int64_t ldx, const void* w, int64_t ldw, void* y, int64_t ldy,
                              const void* rope_cs, int64_t cs_ld, int64_t rot_cols, int head_dim,
                              int32_t* status, void* stream) {
  PE_CHECK_ARG(dtype == PE_BF16 && head_dim == 128,
               "linear + rope: the fused rotation runs on the bf16 tensor-core path with "
               "head_dim 128 (got dtype %d, head_dim %d); use pe_gemm + pe_rope",
               dtype, head_dim);
  if (M == 0) return PE_OK;
  return pe::gemm_tc_rope(M, N, K, x, ldx, w, ldw, y, ldy, rope_cs, cs_ld, rot_cols, status,
                          pe::as_stream(stream));
}

extern "C" int pe_linear_swiglu(int dtype, int64_t M, int64_t I, int64_t K, const void* x,
                                int64_t ldx, const void* w_gu, int64_t ldw, void* gu, int64_t ldgu,
                                void* act, int64_t lda, int algo, int32_t* status, void* stream) {
  PE_CHECK_ARG(M >= 0 && I > 0 && K > 0, "linear + swiglu: bad shape");
  PE_CHECK_ARG(ldgu >= 2 * I && lda >= I, "linear + swiglu: output row stride too small");
  if (M == 0) return PE_OK;
  return pe::gemm_tc_swiglu(dtype, M, I, K, x, ldx, w_gu, ldw, gu, ldgu, act, lda, algo, status,
                            pe::as_stream(stream));
}

extern "C" int pe_linear_swiglu_bwd(int dtype, int64_t M, int64_t I, int64_t K, const void* dy,
                                    int64_t lddy, const void* w, int64_t ldw, const void* gu,
                                    int64_t ldgu, void* dgu, int64_t lddgu, int algo,
                                    int32_t* status, void* stream) {
  PE_CHECK_ARG(M >= 0 && I > 0 && K > 0, "linear + swiglu backward: bad shape");
  PE_CHECK_ARG(lddy >= K && ldw >= I && ldgu >= 2 * I && lddgu >= 2 * I,
               "linear + swiglu backward: row stride too small");
  PE_CHECK_ARG(gu != dgu, "linear + swiglu backward: dgu must not overwrite gate|up");
  if (M == 0) return PE_OK;
  return pe::gemm_tc_swiglu_bwd(dtype, M, I, K, dy, lddy, w, ldw, gu, ldgu, dgu, lddgu, algo,
                                status, pe::as_stream(stream));
}

extern "C" int pe_gemm(int dtype, int64_t M, int64_t N, int64_t K, const void* A, int64_t a_sm,
                       int64_t a_sk, const void* B, int64_t b_sn, int64_t b_sk, void* C,
                       int64_t ldc, int c_dtype, const void* Cin, int64_t ldcin, float alpha,
                       float beta, int algo, int32_t* status, void* stream) {
  return pe::gemm(dtype, M, N, K, A, a_sm, a_sk, B, b_sn, b_sk, C, ldc, c_dtype, Cin, ldcin,
                  alpha, beta, algo, status, pe::as_stream(stream));
}
