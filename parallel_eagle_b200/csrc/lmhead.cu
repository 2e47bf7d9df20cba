// Frozen shared LM head fused with cross-entropy (or soft-target distillation)
// and its input gradient, chunked over the vocabulary (reference
// src/pe/partition.py:113-115, src/pe/drafter.py:123-124).
//
// Pass 1, per vocabulary chunk: Z = h W_c^T on the tensor cores, then an online
// (max, sum-exp) update per row and the label logit.  After the last chunk:
// lse, the loss rows and their sum.  Pass 2, per chunk: recompute Z, form
// G = scale * (softmax - target) rounded to the storage dtype, and accumulate
// dH += G W_c in fp32.  Only one chunk of logits exists at a time, so the
// [rows, vocab] matrix is never stored; the frozen W receives no gradient.
#include "gemm.cuh"

namespace pe {
namespace {

constexpr int64_t kChunk = 8192;
constexpr int kThreads = 256;

__device__ __forceinline__ float block_reduce(float v, bool is_max, float* sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = is_max ? warp_max(v) : warp_sum(v);
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float t = lane < (kThreads / 32) ? sh[lane] : (is_max ? -INFINITY : 0.f);
    t = is_max ? warp_max(t) : warp_sum(t);
    if (lane == 0) sh[32] = t;
  }
  __syncthreads();
  const float r = sh[32];
  __syncthreads();
  return r;
}

// online (max, sumexp) update of each row with this chunk; label logit pick;
// soft targets also carry the teacher's (max, sumexp) and sum_v e^{t-m_t} z_v
template <typename T>
__global__ void __launch_bounds__(kThreads)
stats_kernel(int64_t vc, int64_t v0, const float* __restrict__ Z, const float* __restrict__ Zt,
             int64_t ldz, const int64_t* __restrict__ labels, float* m, float* l, float* zlab,
             float* mt, float* lt, float* szt) {
  __shared__ float sh[33];
  const int64_t r = blockIdx.x;
  const int64_t lab = labels ? labels[r] : 0;
  if (labels && lab < 0) return;  // ignored row (uniform per block)
  const float* z = Z + r * ldz;
  float cmax = -INFINITY;
  for (int64_t c = threadIdx.x; c < vc; c += kThreads) cmax = fmaxf(cmax, round_to<T>(z[c]));
  cmax = block_reduce(cmax, true, sh);
  const float m_old = m[r];
  const float m_new = fmaxf(m_old, cmax);
  float s = 0.f;
  for (int64_t c = threadIdx.x; c < vc; c += kThreads) s += expf(round_to<T>(z[c]) - m_new);
  s = block_reduce(s, false, sh);
  if (Zt) {
    const float* zt = Zt + r * ldz;
    float tmax = -INFINITY;
    for (int64_t c = threadIdx.x; c < vc; c += kThreads) tmax = fmaxf(tmax, round_to<T>(zt[c]));
    tmax = block_reduce(tmax, true, sh);
    const float mt_old = mt[r];
    const float mt_new = fmaxf(mt_old, tmax);
    float st = 0.f, sz = 0.f;
    for (int64_t c = threadIdx.x; c < vc; c += kThreads) {
      const float e = expf(round_to<T>(zt[c]) - mt_new);
      st += e;
      sz += e * round_to<T>(z[c]);
    }
    st = block_reduce(st, false, sh);
    sz = block_reduce(sz, false, sh);
    if (threadIdx.x == 0) {
      const float f = expf(mt_old - mt_new);
      lt[r] = lt[r] * f + st;
      szt[r] = szt[r] * f + sz;
      mt[r] = mt_new;
    }
  }
  if (threadIdx.x == 0) {
    l[r] = l[r] * expf(m_old - m_new) + s;
    m[r] = m_new;
    if (labels && lab >= v0 && lab < v0 + vc) zlab[r] = round_to<T>(z[lab - v0]);
  }
}

// soft-target running stats reset (both rows' (m, l), S_tz, the last rescale factors);
// `flag` (when non-null) clears the overflow word, `run_if` makes the launch conditional
__global__ void soft_init_kernel(int64_t R, float* m, float* l, float* mt, float* lt, float* szt,
                                 float* ks, float* kt, int* flag, const int* run_if) {
  if (run_if != nullptr && *run_if == 0) return;
  if (flag != nullptr && blockIdx.x == 0 && threadIdx.x == 0) *flag = 0;
  for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < R;
       r += (int64_t)gridDim.x * blockDim.x) {
    m[r] = -INFINITY;
    l[r] = 0.f;
    mt[r] = -INFINITY;
    lt[r] = 0.f;
    szt[r] = 0.f;
    ks[r] = 1.f;
    kt[r] = 1.f;
  }
}

__global__ void init_stats_kernel(int64_t R, float* m, float* l, float* zlab, float* mt, float* lt,
                                  float* szt) {
  for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < R;
       r += (int64_t)gridDim.x * blockDim.x) {
    m[r] = -INFINITY;
    l[r] = 0.f;
    zlab[r] = 0.f;
    if (mt) {
      mt[r] = -INFINITY;
      lt[r] = 0.f;
      szt[r] = 0.f;
    }
  }
}

// lse per row, loss rows summed in a fixed order by one block of 1024 threads
constexpr int kFinThreads = 1024;
__global__ void __launch_bounds__(kFinThreads)
finalize_kernel(int64_t R, const int64_t* labels, const float* m, const float* l, const float* zlab,
                const float* mt, const float* lt, const float* szt, float* lse, float* lse_t,
                float* loss_sum) {
  __shared__ float sh[32];
  float acc = 0.f;
  for (int64_t r = threadIdx.x; r < R; r += kFinThreads) {
    if (labels && labels[r] < 0) {
      lse[r] = 0.f;
      continue;
    }
    const float L = m[r] + logf(l[r]);
    lse[r] = L;
    if (mt) {
      lse_t[r] = mt[r] + logf(lt[r]);
      acc += L - szt[r] / lt[r];
    } else {
      acc += L - zlab[r];
    }
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  acc = warp_sum(acc);
  if (lane == 0) sh[warp] = acc;
  __syncthreads();
  if (warp == 0) {
    const float t = warp_sum(sh[lane]);
    if (lane == 0) loss_sum[0] += t;
  }
}

template <typename T>
__global__ void grad_kernel(int64_t R, int64_t vc, int64_t v0, const float* __restrict__ Z,
                            const float* __restrict__ Zt, int64_t ldz,
                            const int64_t* __restrict__ labels, const float* __restrict__ lse,
                            const float* __restrict__ lse_t, float scale, T* __restrict__ G,
                            int64_t ldg) {
  const int64_t total = R * vc;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / vc, c = i - r * vc;
    float g = 0.f;
    const int64_t lab = labels ? labels[r] : 0;
    if (!(labels && lab < 0)) {
      const float p = expf(round_to<T>(Z[r * ldz + c]) - lse[r]);
      float tgt;
      if (Zt)
        tgt = expf(round_to<T>(Zt[r * ldz + c]) - lse_t[r]);
      else
        tgt = (lab == v0 + c) ? 1.f : 0.f;
      g = scale * (p - tgt);
    }
    G[r * ldg + c] = from_f<T>(g);
  }
}

template <typename T>
__global__ void cast2d_kernel(int64_t R, int64_t H, const float* __restrict__ x, T* y, int64_t ldy) {
  const int64_t total = R * H;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / H, c = i - r * H;
    y[r * ldy + c] = from_f<T>(x[i]);
  }
}

int64_t chunk_of(int64_t V) {
  int64_t c = V < kChunk ? V : kChunk;
  return (c + 7) / 8 * 8;
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

struct Layout {
  size_t m, l, zlab, lse, mt, lt, szt, lse_t, Z, Zt, G, dH, total;
};

Layout layout_of(int dtype, int64_t R, int64_t H, int64_t V, int soft) {
  const int64_t vc = chunk_of(V);
  const size_t esz = dtype == PE_F32 ? 4 : 2;
  Layout L{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off += align256(bytes);
    return o;
  };
  L.m = take(4 * R);
  L.l = take(4 * R);
  L.zlab = take(4 * R);
  L.lse = take(4 * R);
  if (soft) {
    L.mt = take(4 * R);
    L.lt = take(4 * R);
    L.szt = take(4 * R);
    L.lse_t = take(4 * R);
  }
  L.Z = take(4 * (size_t)R * vc);
  if (soft) L.Zt = take(4 * (size_t)R * vc);
  L.G = take(esz * (size_t)R * vc);
  L.dH = take(4 * (size_t)R * H);
  L.total = off;
  return L;
}

unsigned grid_for(int64_t n) {
  int64_t g = ceil_div(n, 256);
  const int64_t cap = (int64_t)sm_count() * 16;
  return (unsigned)(g < 1 ? 1 : (g > cap ? cap : g));
}

}  // namespace
}  // namespace pe

// ------------------------------------------------------------------------ //
// Fused path (bf16, hard labels): one logits GEMM per vocabulary chunk, no
// recompute.  Per chunk c:
//   Zc = h W_c^T (bf16) with per-(row, 128-col chunk) (max, sum-exp) from the
//        GEMM epilogue;
//   combine: running (m, l) per row, alpha = exp(m_old - m_new), the label logit,
//        and Zc <- exp(Zc - m_new) in place;
//   dH = Zc W_c + alpha * dH  (fp32, row-scaled accumulate in the GEMM epilogue).
// At the end dh = scale * (dH / l - W[label]): the softmax-minus-one-hot product
// without ever forming the normalised probabilities for the whole vocabulary.
// ------------------------------------------------------------------------ //
namespace pe {
namespace {

// vocabulary rows per logits chunk (default, both paths):
// each chunk ends with a read-modify-write of the fp32 dH accumulator (R x H) in the
// dH GEMM's epilogue, which a 512-wide tile cannot hide, so fewer, longer chunks pay
// it less often.  Measured on the config-2 training step (interleaved A/B, 6 rounds):
// 290.1 ms at 32K against 292.0 at 24K and 293.2 at 16K.
constexpr int64_t kFastChunk = 32768;
// loss rows per group (default).  Groups are equal and a multiple of 128 rows, so the
// ~10240 loss rows of a config-2 sequence run as one group: per chunk the logits GEMM
// has 40 x 32 tiles (17.3 waves of the CTA-pair grid) and the dH GEMM (N = H = 3584)
// 40 x 7 of 512 wide (3.8 waves), with half as many chunk steps as two groups of 5120
// (which left the dH GEMM 1.9 waves).  Measured on the config-2 training step
// (interleaved A/B): 293.4 ms against 294.5 ms for 2 x 5120; 3 x 3456 had been 5-8 %
// slower than 2 x 5120 for the call alone.
constexpr int64_t kRowGroup = 10240;
constexpr int64_t kMaxChunk = 32768;      // hard-label path
constexpr int64_t kMaxChunkSoft = 32768;  // soft-target path (two logits chunks per step)
constexpr int64_t kMaxGroup = 10240;
constexpr int kStatTile = 128;  // columns per (max, sum-exp) pair of the logits GEMM
static_assert(kMaxChunk <= 16 * 256 * 8, "combine_kernel<16> covers at most 32K columns");
static_assert(kMaxChunkSoft <= 512 * 64, "combine_soft_kernel<512> covers at most 32K columns");

// Rows of the loss are processed in groups, which bounds the logits chunk (group x
// chunk bf16) held between the logits GEMM, the combine pass and the dH GEMM.  ``algo`` bits 8-15 override the chunk (units of
// 1024 vocabulary rows) and bits 16-23 the group (units of 256 loss rows).
struct FastPlan {
  int64_t vc, rg;
  int logits_bn, dh_bn;  // pair tile widths (0: the GEMMs' own choice)
};

// algo bits 24-25 / 26-27: logits / dH GEMM pair tile width (1: 256, 2: 512, 0: automatic)
FastPlan fast_plan_of(int64_t R, int64_t V, int algo, int64_t max_chunk) {
  int64_t vc = ((algo >> 8) & 0xff) ? ((algo >> 8) & 0xff) * 1024 : kFastChunk;
  int64_t rg = ((algo >> 16) & 0xff) ? ((algo >> 16) & 0xff) * 256 : kRowGroup;
  vc = vc > max_chunk ? max_chunk : vc;
  rg = rg > kMaxGroup ? kMaxGroup : rg;
  if (V < vc) vc = (V + 7) / 8 * 8;
  if (R <= rg) {
    rg = R;
  } else {  // equal groups, each a multiple of the 128-row tile
    const int64_t ng = (R + rg - 1) / rg;
    rg = ((R + ng - 1) / ng + 127) / 128 * 128;
  }
  const int lb = (algo >> 24) & 3, db = (algo >> 26) & 3;
  return {vc, rg, lb == 1 ? 256 : lb == 2 ? 512 : 0, db == 1 ? 256 : db == 2 ? 512 : 0};
}

struct FastLayout {
  size_t m, l, zlab, lse, alpha, keep[3], keep_last, m0, flag, stats[2], Z[2], dH, total;
};

// sized for the largest plan any ``algo`` can select, so one workspace serves all
FastLayout fast_layout_of(int64_t R, int64_t H, int64_t V) {
  const int64_t vc = V < kMaxChunk ? (V + 7) / 8 * 8 : kMaxChunk;
  const int64_t rg = R < kMaxGroup ? R : kMaxGroup;
  const int64_t nt = (vc + kStatTile - 1) / kStatTile;
  FastLayout L{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off += align256(bytes);
    return o;
  };
  L.m = take(4 * R);
  L.l = take(4 * R);
  L.zlab = take(4 * R);
  L.lse = take(4 * R);
  L.alpha = take(4 * R);
  for (int b = 0; b < 3; ++b) L.keep[b] = take(4 * R);
  L.keep_last = take(4 * R);
  L.m0 = take(4 * R);
  L.flag = take(4);
  for (int b = 0; b < 2; ++b) {  // double-buffered: chunk j+1's logits overlap chunk j
    L.stats[b] = take(8 * (size_t)rg * nt);
    L.Z[b] = take(2 * (size_t)rg * vc);
  }
  L.dH = take(4 * (size_t)R * H);
  L.total = off;
  return L;
}

// per row: fold this chunk's tile stats into (m, l), record the rescale factor,
// pick the label logit, and overwrite the chunk's logits with exp(z - m_new).
// Warp 0 folds the (at most 256) tile stats, lane l taking tiles l, l + 32, ...
template <int kPer>  // 16-byte loads per thread: vc <= kPer * 256 * 8
__global__ void __launch_bounds__(256)
combine_kernel(int64_t R, int64_t vc, int64_t v0, int nt, int stats_ld,
               const float2* __restrict__ stats, __nv_bfloat16* __restrict__ Z, int64_t ldz,
               const int64_t* __restrict__ labels, float* m, float* l, float* zlab, float* alpha,
               const int* run_if) {
  // a conditional launch (the recomputation after an overflow) has a small grid, so
  // that skipping it costs little: blocks walk rows r = blockIdx.x, + gridDim.x, ...
  if (run_if != nullptr && *run_if == 0) return;
  __shared__ float s_mnew;
  for (int64_t r = blockIdx.x; r < R; r += gridDim.x) {
    const int64_t lab = labels[r];
    __nv_bfloat16* z = Z + r * ldz;
    // every thread's share of the row (kPer pieces of 16 B) is loaded before the stats
    // fold, so all of a row's loads are in flight together: a load-exp-store loop over
    // a row rewritten in place cannot hoist a load above the previous store, and paid
    // one DRAM round trip per piece
    uint4 buf[kPer];
#pragma unroll
    for (int q = 0; q < kPer; ++q) {
      const int64_t c = ((int64_t)threadIdx.x + (int64_t)q * 256) * 8;
      if (c < vc) buf[q] = *reinterpret_cast<const uint4*>(z + c);
    }
    if (threadIdx.x < 32) {
      const int lane = threadIdx.x;
      const float2* st = stats + r * stats_ld;
      const float m_old = m[r];
      // nt <= kPer * 2048 / kStatTile: lane takes tiles lane, lane + 32, ...
      constexpr int kSv = kPer * 2048 / kStatTile / 32;
      float2 sv[kSv];
      float lm = -INFINITY;
#pragma unroll
      for (int q = 0; q < kSv; ++q) {
        const int t = lane + 32 * q;
        sv[q] = t < nt ? st[t] : make_float2(-INFINITY, 0.f);
        lm = fmaxf(lm, sv[q].x);
      }
      const float mn = fmaxf(m_old, warp_max(lm));
      float part = 0.f;
#pragma unroll
      for (int q = 0; q < kSv; ++q)
        if (sv[q].x != -INFINITY) part += sv[q].y * expf(sv[q].x - mn);
      const float tile_sum = warp_sum(part);
      if (lane == 0) {
        const float keep = m_old == -INFINITY ? 0.f : expf(m_old - mn);
        l[r] = l[r] * keep + tile_sum;
        alpha[r] = keep;
        m[r] = mn;
        if (lab >= v0 && lab < v0 + vc) zlab[r] = __bfloat162float(z[lab - v0]);
        s_mnew = mn;
      }
    }
    __syncthreads();
    const float mn = s_mnew;
    const bool ignored = lab < 0;
#pragma unroll
    for (int q = 0; q < kPer; ++q) {
      const int64_t c = ((int64_t)threadIdx.x + (int64_t)q * 256) * 8;
      if (c < vc) {
        uint4 u = buf[q];
        __nv_bfloat162* h2 = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          float2 f = __bfloat1622float2(h2[i]);
          f.x = ignored ? 0.f : __expf(f.x - mn);
          f.y = ignored ? 0.f : __expf(f.y - mn);
          h2[i] = __floats2bfloat162_rn(f.x, f.y);
        }
        *reinterpret_cast<uint4*>(z + c) = u;
      }
    }
    __syncthreads();  // s_mnew is rewritten for the next row
  }
}

// running stats reset; `flag` (when non-null) clears the single-pass overflow word
__global__ void fast_init_kernel(int64_t R, float* m, float* l, float* zlab, float* keep_last,
                                 int* flag, const int* run_if) {
  if (run_if != nullptr && *run_if == 0) return;
  if (flag != nullptr && blockIdx.x == 0 && threadIdx.x == 0) *flag = 0;
  for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < R;
       r += (int64_t)gridDim.x * blockDim.x) {
    m[r] = -INFINITY;
    l[r] = 0.f;
    zlab[r] = 0.f;
    keep_last[r] = 1.f;
  }
}

// First chunk of a row group (one warp per row): the row maximum m0 and l = sum of
// e^(z - m0) from the chunk's (tile max, sum e^(z - tile max)) pairs, and the label
// logit when the label falls in the chunk.  keep = 1: the next chunk's exponentials
// are taken relative to m0, the reference of this chunk's.
__global__ void __launch_bounds__(256)
fold_first_kernel(int64_t R, int64_t vc, int nt, int stats_ld, const float2* __restrict__ stats,
                  const __nv_bfloat16* __restrict__ Z, int64_t ldz,
                  const int64_t* __restrict__ labels, float* m, float* l, float* m0, float* zlab,
                  float* keep, float* keep_last) {
  const int lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (r >= R) return;
  const float2* st = stats + r * stats_ld;
  float lm = -INFINITY;
  for (int t = lane; t < nt; t += 32) lm = fmaxf(lm, st[t].x);
  const float mx = warp_max(lm);
  float part = 0.f;
  for (int t = lane; t < nt; t += 32) {
    const float2 v = st[t];
    if (v.x != -INFINITY) part += v.y * expf(v.x - mx);
  }
  const float sum = warp_sum(part);
  if (lane == 0) {
    m[r] = mx;
    m0[r] = mx;
    l[r] = sum;
    keep[r] = 1.f;
    keep_last[r] = 1.f;
    const int64_t lab = labels ? labels[r] : -1;  // soft targets: no labels
    if (lab >= 0 && lab < vc) zlab[r] = __bfloat162float(Z[r * ldz + lab]);
  }
}

// First chunk of a row group, in place: Z <- e^(z - m0) (0 for an ignored row).  All
// of a thread's 16-byte pieces of the row are loaded before any is rewritten.
template <int kPer>
__global__ void __launch_bounds__(256)
exp_first_kernel(int64_t vc, __nv_bfloat16* __restrict__ Z, int64_t ldz,
                 const int64_t* __restrict__ labels, const float* __restrict__ m0) {
  const int64_t r = blockIdx.x;
  __nv_bfloat16* z = Z + r * ldz;
  const bool ignored = labels != nullptr && labels[r] < 0;
  const float mx = m0[r];
  uint4 buf[kPer];
#pragma unroll
  for (int q = 0; q < kPer; ++q) {
    const int64_t c = ((int64_t)threadIdx.x + (int64_t)q * 256) * 8;
    if (c < vc) buf[q] = *reinterpret_cast<const uint4*>(z + c);
  }
#pragma unroll
  for (int q = 0; q < kPer; ++q) {
    const int64_t c = ((int64_t)threadIdx.x + (int64_t)q * 256) * 8;
    if (c < vc) {
      uint4 u = buf[q];
      __nv_bfloat162* h2 = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float2 f = __bfloat1622float2(h2[i]);
        f.x = ignored ? 0.f : __expf(f.x - mx);
        f.y = ignored ? 0.f : __expf(f.y - mx);
        h2[i] = __floats2bfloat162_rn(f.x, f.y);
      }
      *reinterpret_cast<uint4*>(z + c) = u;
    }
  }
}

// Later chunk (one warp per row): its exponentials were taken relative to the running
// maximum m_old, so with M = max(m_old, tile maxima) and keep = e^(m_old - M):
//   l <- l keep + sum_t S_t keep   (S_t: the tile's sum of e^(z - m_old))
// each S_t scaled before the sum, so the sum stays in range.  keep is also the factor
// the next chunk's dH accumulation applies to the running dH, and the last chunk's
// keep the factor the final dH applies (keep_last).
__global__ void __launch_bounds__(256)
fold_kernel(int64_t R, int nt, int stats_ld, const float2* __restrict__ stats, float* m, float* l,
            float* keep, float* keep_last) {
  const int lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (r >= R) return;
  const float2* st = stats + r * stats_ld;
  const float m_old = m[r];
  float lm = -INFINITY;
  for (int t = lane; t < nt; t += 32) lm = fmaxf(lm, st[t].x);
  const float mx = fmaxf(m_old, warp_max(lm));
  const float kp = expf(m_old - mx);
  float part = 0.f;
  for (int t = lane; t < nt; t += 32) part += st[t].y * kp;
  const float sum = warp_sum(part);
  if (lane == 0) {
    m[r] = mx;
    l[r] = l[r] * kp + sum;
    keep[r] = kp;
    keep_last[r] = kp;
  }
}

// dh = scale * (dH keep_last / l - W[label])
__global__ void fast_dh_kernel(int64_t R, int64_t H, const float* __restrict__ dH,
                               const float* __restrict__ l, const float* __restrict__ keep_last,
                               const int64_t* __restrict__ labels,
                               const __nv_bfloat16* __restrict__ W, float scale,
                               __nv_bfloat16* __restrict__ dh, int64_t lddh) {
  const int64_t total = R * H / 8;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = i * 8;
    const int64_t r = e / H, c = e - r * H;
    const int64_t lab = labels[r];
    uint4 out = make_uint4(0, 0, 0, 0);
    if (lab >= 0) {
      const float inv = keep_last[r] / l[r];
      const float4 a = reinterpret_cast<const float4*>(dH + e)[0];
      const float4 b = reinterpret_cast<const float4*>(dH + e)[1];
      const uint4 wu = *reinterpret_cast<const uint4*>(W + lab * H + c);
      const __nv_bfloat162* w2 = reinterpret_cast<const __nv_bfloat162*>(&wu);
      const float2 w0 = __bfloat1622float2(w2[0]), w1 = __bfloat1622float2(w2[1]);
      const float2 w2f = __bfloat1622float2(w2[2]), w3 = __bfloat1622float2(w2[3]);
      __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&out);
      o2[0] = __floats2bfloat162_rn(scale * (a.x * inv - w0.x), scale * (a.y * inv - w0.y));
      o2[1] = __floats2bfloat162_rn(scale * (a.z * inv - w1.x), scale * (a.w * inv - w1.y));
      o2[2] = __floats2bfloat162_rn(scale * (b.x * inv - w2f.x), scale * (b.y * inv - w2f.y));
      o2[3] = __floats2bfloat162_rn(scale * (b.z * inv - w3.x), scale * (b.w * inv - w3.y));
    }
    *reinterpret_cast<uint4*>(dh + r * lddh + c) = out;
  }
}

bool fast_eligible(int dtype, int64_t H, int64_t V, const void* h, int64_t ldh, const void* W,
                   const void* teacher, void* dh, int64_t lddh, int algo) {
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  return dtype == PE_BF16 && teacher == nullptr && algo != PE_ALGO_SIMT && H % 8 == 0 &&
         V % 8 == 0 && ldh % 8 == 0 && lddh % 8 == 0 && a16(h) && a16(W) && a16(dh);
}

// Software pipeline over (row group, vocabulary chunk) steps t.  The first chunk of a
// group runs in two passes: the logits GEMM stores the bf16 logits with per-tile
// (max, sum e^(z - max)) pairs, a fold gives the row maximum m0, and the side stream
// rewrites the chunk as e^(z - m0) before the dH GEMM.  Every later chunk is one pass:
// its logits GEMM writes P = e^(z - m) directly, m the running maximum of the earlier
// chunks (no bf16 logits are stored or re-read), and a fold on the same stream updates
// (m, l) before the next chunk's GEMM reads m.  The dH GEMM of chunk t (side stream)
// rescales the running dH by e^(m_{t-2} - m_{t-1}) (the fold of chunk t - 1) and adds
// P W; the final dH is rescaled once more by the last fold's factor.  So one GEMM's last
// partial wave, the fold and the first chunk's rewrite overlap the other GEMM.  Z, the
// stats and the per-chunk factors are double- / triple-buffered: the logits GEMM of
// step t waits for the dH GEMM of step t-2, which read the factors of step t-3.
// If some logit exceeds its row's running maximum by more than e^64 allows, the
// epilogue sets an overflow word and every pass of the classic two-pass algorithm
// below runs as well (each launch returns at once when the word is 0), recomputing the
// whole call; the loss and dh always come from the pass that ran last.
int lmhead_fast(int64_t R, int64_t H, int64_t V, const void* h, int64_t ldh, const void* W,
                const int64_t* labels, float grad_scale, void* dh, int64_t lddh, float* loss_sum,
                uint8_t* ws, int algo, int* status, cudaStream_t st) {
  const FastLayout L = fast_layout_of(R, H, V);
  const FastPlan P = fast_plan_of(R, V, algo, kMaxChunk);
  float* m = (float*)(ws + L.m);
  float* l = (float*)(ws + L.l);
  float* zlab = (float*)(ws + L.zlab);
  float* lse = (float*)(ws + L.lse);
  float* alpha = (float*)(ws + L.alpha);
  float* keep[3] = {(float*)(ws + L.keep[0]), (float*)(ws + L.keep[1]), (float*)(ws + L.keep[2])};
  float* keep_last = (float*)(ws + L.keep_last);
  float* m0 = (float*)(ws + L.m0);
  int* flag = (int*)(ws + L.flag);
  float2* stats[2] = {(float2*)(ws + L.stats[0]), (float2*)(ws + L.stats[1])};
  __nv_bfloat16* Z[2] = {(__nv_bfloat16*)(ws + L.Z[0]), (__nv_bfloat16*)(ws + L.Z[1])};
  float* dH = (float*)(ws + L.dH);
  const int64_t VC = P.vc;
  const int nt_max = (int)((VC + kStatTile - 1) / kStatTile);
  // 8 loads of 16 B per thread cover chunks up to 16K columns, 16 up to 32K (a single
  // width would hold 16 in registers and halve the blocks per SM)
  auto exp_first = VC <= 16384 ? exp_first_kernel<8> : exp_first_kernel<16>;
  auto combine = VC <= 16384 ? combine_kernel<8> : combine_kernel<16>;
  cudaStream_t side = side_stream(0);
  cudaEvent_t ev_fork = pool_event(0), ev_join = pool_event(1);
  cudaEvent_t ev_logits[2] = {pool_event(2), pool_event(3)};
  cudaEvent_t ev_dh[2] = {pool_event(4), pool_event(5)};
  if (!side || !ev_fork || !ev_join || !ev_logits[0] || !ev_logits[1] || !ev_dh[0] || !ev_dh[1]) {
    set_error("lmhead_ce: could not create the side stream or its events");
    return PE_ERR_CUDA;
  }
  // algo bit 28: the two-pass algorithm for every chunk (kept for comparison)
  const bool two_pass = (algo >> 28) & 1;
  fast_init_kernel<<<grid_for(R), 256, 0, st>>>(R, m, l, zlab, keep_last, flag, nullptr);
  PE_LAUNCHED();
  PE_CUDA_TRY(cudaEventRecord(ev_fork, st));
  PE_CUDA_TRY(cudaStreamWaitEvent(side, ev_fork, 0));
  int64_t t = 0;
  for (int64_t r0 = 0; r0 < R; r0 += P.rg) {
    const int64_t rg = (R - r0) < P.rg ? (R - r0) : P.rg;
    const void* hg = (const __nv_bfloat16*)h + r0 * ldh;
    float* dHg = dH + r0 * H;
    const unsigned fold_grid = (unsigned)((rg + 7) / 8);
    for (int64_t v0 = 0; v0 < V; v0 += VC, ++t) {
      const int b = (int)(t & 1);
      const int64_t vc = (V - v0) < VC ? (V - v0) : VC;
      const int nt = (int)((vc + kStatTile - 1) / kStatTile);
      const __nv_bfloat16* Wc = (const __nv_bfloat16*)W + v0 * H;
      float* kt = keep[t % 3] + r0;
      if (t >= 2) PE_CUDA_TRY(cudaStreamWaitEvent(st, ev_dh[b], 0));
      int rc;
      if (two_pass) {
        rc = gemm_tc_logits_stats(rg, vc, H, hg, ldh, Wc, H, Z[b], VC, stats[b], nt_max, status,
                                  st, P.logits_bn);
        if (rc) return rc;
        PE_CUDA_TRY(cudaEventRecord(ev_logits[b], st));
        PE_CUDA_TRY(cudaStreamWaitEvent(side, ev_logits[b], 0));
        combine<<<(unsigned)rg, 256, 0, side>>>(rg, vc, v0, nt, nt_max, stats[b], Z[b], VC,
                                                labels + r0, m + r0, l + r0, zlab + r0,
                                                alpha + r0, nullptr);
        PE_LAUNCHED();
        rc = gemm_tc_rowscale_acc(rg, H, vc, Z[b], VC, Wc, H, dHg, H, v0 > 0 ? dHg : nullptr,
                                  alpha + r0, status, side, P.dh_bn);
      } else if (v0 == 0) {
        rc = gemm_tc_logits_stats(rg, vc, H, hg, ldh, Wc, H, Z[b], VC, stats[b], nt_max, status,
                                  st, P.logits_bn);
        if (rc) return rc;
        fold_first_kernel<<<fold_grid, 256, 0, st>>>(rg, vc, nt, nt_max, stats[b], Z[b], VC,
                                                     labels + r0, m + r0, l + r0, m0 + r0,
                                                     zlab + r0, kt, keep_last + r0);
        PE_LAUNCHED();
        PE_CUDA_TRY(cudaEventRecord(ev_logits[b], st));
        PE_CUDA_TRY(cudaStreamWaitEvent(side, ev_logits[b], 0));
        exp_first<<<(unsigned)rg, 256, 0, side>>>(vc, Z[b], VC, labels + r0, m0 + r0);
        PE_LAUNCHED();
        rc = gemm_tc_rowscale_acc(rg, H, vc, Z[b], VC, Wc, H, dHg, H, nullptr, kt, status, side,
                                  P.dh_bn);
      } else {
        rc = gemm_tc_logits_pexp(rg, vc, H, hg, ldh, Wc, H, Z[b], VC, stats[b], nt_max, m + r0,
                                 labels + r0, v0, zlab + r0, flag, status, st, P.logits_bn);
        if (rc) return rc;
        fold_kernel<<<fold_grid, 256, 0, st>>>(rg, nt, nt_max, stats[b], m + r0, l + r0, kt,
                                               keep_last + r0);
        PE_LAUNCHED();
        PE_CUDA_TRY(cudaEventRecord(ev_logits[b], st));
        PE_CUDA_TRY(cudaStreamWaitEvent(side, ev_logits[b], 0));
        rc = gemm_tc_rowscale_acc(rg, H, vc, Z[b], VC, Wc, H, dHg, H, dHg, keep[(t + 2) % 3] + r0,
                                  status, side, P.dh_bn);
      }
      if (rc) return rc;
      PE_CUDA_TRY(cudaEventRecord(ev_dh[b], side));
    }
  }
  PE_CUDA_TRY(cudaEventRecord(ev_join, side));
  PE_CUDA_TRY(cudaStreamWaitEvent(st, ev_join, 0));
  // recomputation after an overflow: the classic two-pass algorithm on one stream, every
  // launch conditional on the overflow word
  if (!two_pass) {
    fast_init_kernel<<<grid_for(R), 256, 0, st>>>(R, m, l, zlab, keep_last, nullptr, flag);
    PE_LAUNCHED();
  }
  for (int64_t r0 = 0; r0 < R && !two_pass; r0 += P.rg) {
    const int64_t rg = (R - r0) < P.rg ? (R - r0) : P.rg;
    const void* hg = (const __nv_bfloat16*)h + r0 * ldh;
    float* dHg = dH + r0 * H;
    for (int64_t v0 = 0; v0 < V; v0 += VC) {
      const int64_t vc = (V - v0) < VC ? (V - v0) : VC;
      const int nt = (int)((vc + kStatTile - 1) / kStatTile);
      const __nv_bfloat16* Wc = (const __nv_bfloat16*)W + v0 * H;
      int rc = gemm_tc_logits_stats(rg, vc, H, hg, ldh, Wc, H, Z[0], VC, stats[0], nt_max, status,
                                    st, P.logits_bn, flag);
      if (rc) return rc;
      combine<<<(unsigned)(rg < 2 * sm_count() ? rg : 2 * sm_count()), 256, 0, st>>>(
          rg, vc, v0, nt, nt_max, stats[0], Z[0], VC, labels + r0, m + r0, l + r0, zlab + r0,
          alpha + r0, flag);
      PE_LAUNCHED();
      rc = gemm_tc_rowscale_acc(rg, H, vc, Z[0], VC, Wc, H, dHg, H, v0 > 0 ? dHg : nullptr,
                                alpha + r0, status, st, P.dh_bn, flag);
      if (rc) return rc;
    }
  }
  finalize_kernel<<<1, kFinThreads, 0, st>>>(R, labels, m, l, zlab, nullptr, nullptr, nullptr, lse,
                                          nullptr, loss_sum);
  PE_LAUNCHED();
  fast_dh_kernel<<<grid_for(R * H / 8), 256, 0, st>>>(R, H, dH, l, keep_last, labels,
                                                      (const __nv_bfloat16*)W, grad_scale,
                                                      (__nv_bfloat16*)dh, lddh);
  PE_LAUNCHED();
  return PE_OK;
}

// ------------------------------------------------------------------------ //
// Fused soft-target path (bf16, teacher rows t_r): per (row group, chunk) step
//   Zs = h W_c^T, Zt = t W_c^T (bf16, per-128-column (max, sum-exp) stats from the
//   GEMM epilogues);
//   combine_soft: running (m_s, l_s) and (m_t, l_t), rescale factors alpha_s /
//   alpha_t, S_tz = sum_v e^{t_v - m_t} z_v (online), and in place
//   Zs <- e^{z - m_s}, Zt <- e^{t - m_t};
//   dH_s = Zs W_c + alpha_s dH_s,  dH_t = Zt W_c + alpha_t dH_t  (fp32).
// loss_r = (m_s + ln l_s) - S_tz / l_t ;  dh = scale (dH_s / l_s - dH_t / l_t).
// Four GEMMs per chunk, every logits chunk bf16 and L2-sized, one pass over W.
// ------------------------------------------------------------------------ //
struct SoftLayout {
  size_t m, l, zlab, lse, alpha, mt, lt, szt, alpha_t, lse_t, keep_s[3], keep_t[3], keep_last_s,
      keep_last_t, m0_s, m0_t, flag, stats_s[2], stats_t[2], Zs[2], Zt[2], dHs, dHt, total;
};

SoftLayout soft_layout_of(int64_t R, int64_t H, int64_t V) {
  const int64_t vc = V < kMaxChunkSoft ? (V + 7) / 8 * 8 : kMaxChunkSoft;
  const int64_t rg = R < kMaxGroup ? R : kMaxGroup;
  const int64_t nt = (vc + kStatTile - 1) / kStatTile;
  SoftLayout L{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off += align256(bytes);
    return o;
  };
  L.m = take(4 * R);
  L.l = take(4 * R);
  L.zlab = take(4 * R);
  L.lse = take(4 * R);
  L.alpha = take(4 * R);
  L.mt = take(4 * R);
  L.lt = take(4 * R);
  L.szt = take(4 * R);
  L.alpha_t = take(4 * R);
  L.lse_t = take(4 * R);
  for (int b = 0; b < 3; ++b) {
    L.keep_s[b] = take(4 * R);
    L.keep_t[b] = take(4 * R);
  }
  L.keep_last_s = take(4 * R);
  L.keep_last_t = take(4 * R);
  L.m0_s = take(4 * R);
  L.m0_t = take(4 * R);
  L.flag = take(4);
  for (int b = 0; b < 2; ++b) {
    L.stats_s[b] = take(8 * (size_t)rg * nt);
    L.stats_t[b] = take(8 * (size_t)rg * nt);
    L.Zs[b] = take(2 * (size_t)rg * vc);
    L.Zt[b] = take(2 * (size_t)rg * vc);
  }
  L.dHs = take(4 * (size_t)R * H);
  L.dHt = take(4 * (size_t)R * H);
  L.total = off;
  return L;
}

// fold one chunk's tile stats (at most 32 kSv tiles, lane takes tiles lane + 32 q) into
// a running (m, l); returns the new maximum, writes l and the rescale factor
template <int kSv>
__device__ __forceinline__ float fold_stats(const float2* st, int nt, float* m, float* l,
                                            float* alpha, int lane) {
  float2 sv[kSv];
  float lm = -INFINITY;
#pragma unroll
  for (int q = 0; q < kSv; ++q) {
    const int t = lane + 32 * q;
    sv[q] = t < nt ? st[t] : make_float2(-INFINITY, 0.f);
    lm = fmaxf(lm, sv[q].x);
  }
  const float m_old = *m;
  const float mn = fmaxf(m_old, warp_max(lm));
  float part = 0.f;
#pragma unroll
  for (int q = 0; q < kSv; ++q)
    if (sv[q].x != -INFINITY) part += sv[q].y * expf(sv[q].x - mn);
  const float tile_sum = warp_sum(part);
  const float keep = m_old == -INFINITY ? 0.f : expf(m_old - mn);
  if (lane == 0) {
    *l = *l * keep + tile_sum;
    *alpha = keep;
    *m = mn;
  }
  return __shfl_sync(0xffffffffu, mn, 0);
}

// kT threads per row (256 or 512), eight 16-byte pieces of each row per thread: chunks
// of up to kT * 64 columns (16K or 32K).  Blocks walk rows r = blockIdx.x, + gridDim.x,
// ... (the conditional recomputation after an overflow runs with a small grid and
// returns at once unless *run_if is set).
template <int kT>
__global__ void __launch_bounds__(kT)
combine_soft_kernel(int64_t R, int64_t vc, int nt, int stats_ld,
                    const float2* __restrict__ stats_s, const float2* __restrict__ stats_t,
                    __nv_bfloat16* __restrict__ Zs, __nv_bfloat16* __restrict__ Zt, int64_t ldz,
                    float* m, float* l, float* alpha, float* mt, float* lt, float* szt,
                    float* alpha_t, const int* run_if) {
  if (run_if != nullptr && *run_if == 0) return;
  __shared__ float s_m[2];
  constexpr int kWarps = kT / 32;
  constexpr int kSv = kT * 64 / kStatTile / 32;  // tile stats per lane
  __shared__ float s_red[kWarps];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int64_t r = blockIdx.x; r < R; r += gridDim.x) {
    __nv_bfloat16* zs = Zs + r * ldz;
    __nv_bfloat16* zt = Zt + r * ldz;
    // the thread's share of both rows is loaded before the stats folds (all loads of
    // the rows in flight together; see combine_kernel)
    constexpr int kPer = 8;
    uint4 bs[kPer], bt[kPer];
#pragma unroll
    for (int q = 0; q < kPer; ++q) {
      const int64_t c = ((int64_t)threadIdx.x + (int64_t)q * kT) * 8;
      if (c < vc) {
        bs[q] = *reinterpret_cast<const uint4*>(zs + c);
        bt[q] = *reinterpret_cast<const uint4*>(zt + c);
      }
    }
    if (warp == 0) {
      const float ms = fold_stats<kSv>(stats_s + r * stats_ld, nt, m + r, l + r, alpha + r, lane);
      if (lane == 0) s_m[0] = ms;
    } else if (warp == 1) {
      const float mtn =
          fold_stats<kSv>(stats_t + r * stats_ld, nt, mt + r, lt + r, alpha_t + r, lane);
      if (lane == 0) s_m[1] = mtn;
    }
    __syncthreads();
    const float ms = s_m[0], mtn = s_m[1];
    float acc = 0.f;
#pragma unroll
    for (int q = 0; q < kPer; ++q) {
      const int64_t c = ((int64_t)threadIdx.x + (int64_t)q * kT) * 8;
      if (c >= vc) continue;
      uint4 us = bs[q];
      uint4 ut = bt[q];
      __nv_bfloat162* hs = reinterpret_cast<__nv_bfloat162*>(&us);
      __nv_bfloat162* ht = reinterpret_cast<__nv_bfloat162*>(&ut);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 z = __bfloat1622float2(hs[i]), t = __bfloat1622float2(ht[i]);
        const float p0 = __expf(t.x - mtn), p1 = __expf(t.y - mtn);
        acc += p0 * z.x + p1 * z.y;
        hs[i] = __floats2bfloat162_rn(__expf(z.x - ms), __expf(z.y - ms));
        ht[i] = __floats2bfloat162_rn(p0, p1);
      }
      *reinterpret_cast<uint4*>(zs + c) = us;
      *reinterpret_cast<uint4*>(zt + c) = ut;
    }
    acc = warp_sum(acc);
    if (lane == 0) s_red[warp] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
      float t = 0.f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) t += s_red[w];
      szt[r] = szt[r] * alpha_t[r] + t;
    }
    __syncthreads();  // s_m / s_red are rewritten for the next row
  }
}

// One-pass soft targets (one warp per row): szt = sum_v e^(t_v - m_t) z_v, taken as
// h . (dH_t keep_last_t), since dH_t = sum_v e^(t_v - m_t') W_v and z_v = h . W_v -- the
// student's logits themselves are never stored.
__global__ void __launch_bounds__(256)
soft_tz_kernel(int64_t R, int64_t H, const __nv_bfloat16* __restrict__ h, int64_t ldh,
               const float* __restrict__ dHt, const float* __restrict__ keep_last_t,
               float* __restrict__ szt) {
  const int lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (r >= R) return;
  const __nv_bfloat16* hr = h + r * ldh;
  const float* dr = dHt + r * H;
  float acc = 0.f;
  for (int64_t c = (int64_t)lane * 8; c < H; c += 256) {
    const uint4 u = *reinterpret_cast<const uint4*>(hr + c);
    const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&u);
    const float4 a = reinterpret_cast<const float4*>(dr + c)[0];
    const float4 b = reinterpret_cast<const float4*>(dr + c)[1];
    const float2 h0 = __bfloat1622float2(h2[0]), h1 = __bfloat1622float2(h2[1]);
    const float2 h2f = __bfloat1622float2(h2[2]), h3 = __bfloat1622float2(h2[3]);
    acc += h0.x * a.x + h0.y * a.y + h1.x * a.z + h1.y * a.w;
    acc += h2f.x * b.x + h2f.y * b.y + h3.x * b.z + h3.y * b.w;
  }
  acc = warp_sum(acc);
  if (lane == 0) szt[r] = acc * keep_last_t[r];
}

// dh = scale * (dH_s ks / l_s - dH_t kt / l_t), ks / kt the last chunk's rescale factors
// (1 after the two-pass algorithm)
__global__ void soft_dh_kernel(int64_t R, int64_t H, const float* __restrict__ dHs,
                               const float* __restrict__ dHt, const float* __restrict__ l,
                               const float* __restrict__ lt, const float* __restrict__ ks,
                               const float* __restrict__ kt, float scale,
                               __nv_bfloat16* __restrict__ dh, int64_t lddh) {
  const int64_t total = R * H / 8;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = i * 8;
    const int64_t r = e / H, c = e - r * H;
    const float is = ks[r] / l[r], it = kt[r] / lt[r];
    float o[8];
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const float4 a = reinterpret_cast<const float4*>(dHs + e)[q];
      const float4 b = reinterpret_cast<const float4*>(dHt + e)[q];
      o[4 * q] = scale * (a.x * is - b.x * it);
      o[4 * q + 1] = scale * (a.y * is - b.y * it);
      o[4 * q + 2] = scale * (a.z * is - b.z * it);
      o[4 * q + 3] = scale * (a.w * is - b.w * it);
    }
    uint4 out;
    __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&out);
#pragma unroll
    for (int k = 0; k < 4; ++k) o2[k] = __floats2bfloat162_rn(o[2 * k], o[2 * k + 1]);
    *reinterpret_cast<uint4*>(dh + r * lddh + c) = out;
  }
}

bool soft_fast_eligible(int dtype, int64_t H, int64_t V, const void* h, int64_t ldh,
                        const void* W, const void* teacher, int64_t ldt, void* dh, int64_t lddh,
                        int algo) {
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  return dtype == PE_BF16 && teacher != nullptr && algo != PE_ALGO_SIMT && H % 8 == 0 &&
         V % 8 == 0 && ldh % 8 == 0 && ldt % 8 == 0 && lddh % 8 == 0 && a16(h) && a16(W) &&
         a16(teacher) && a16(dh);
}

// Same two-stream chunk pipeline as lmhead_fast, with the teacher's logits GEMM next
// to the student's and two dH accumulations on the side stream.  As there, a row
// group's first chunk is two-pass (both GEMMs store bf16 logits, two folds, two
// in-place rewrites as e^(z - m0)) and every later chunk one-pass (both GEMMs write
// e^(z - m) / e^(t - m_t) directly, two folds); the loss's S_tz = sum_v e^(t_v - m_t)
// z_v is h . dH_t at the end (soft_tz_kernel).  An overflow of either running maximum
// recomputes the call two-pass (the combine pass, which also accumulates S_tz from the
// stored logits); algo bit 28 runs every chunk that way.
int lmhead_fast_soft(int64_t R, int64_t H, int64_t V, const void* h, int64_t ldh, const void* W,
                     const void* teacher, int64_t ldt, float grad_scale, void* dh, int64_t lddh,
                     float* loss_sum, uint8_t* ws, int algo, int* status, cudaStream_t st) {
  const SoftLayout L = soft_layout_of(R, H, V);
  const FastPlan P = fast_plan_of(R, V, algo, kMaxChunkSoft);
  float* m = (float*)(ws + L.m);
  float* l = (float*)(ws + L.l);
  float* zlab = (float*)(ws + L.zlab);
  float* lse = (float*)(ws + L.lse);
  float* alpha = (float*)(ws + L.alpha);
  float* mt = (float*)(ws + L.mt);
  float* lt = (float*)(ws + L.lt);
  float* szt = (float*)(ws + L.szt);
  float* alpha_t = (float*)(ws + L.alpha_t);
  float* lse_t = (float*)(ws + L.lse_t);
  float* ks[3] = {(float*)(ws + L.keep_s[0]), (float*)(ws + L.keep_s[1]),
                  (float*)(ws + L.keep_s[2])};
  float* kt[3] = {(float*)(ws + L.keep_t[0]), (float*)(ws + L.keep_t[1]),
                  (float*)(ws + L.keep_t[2])};
  float* ks_last = (float*)(ws + L.keep_last_s);
  float* kt_last = (float*)(ws + L.keep_last_t);
  float* m0s = (float*)(ws + L.m0_s);
  float* m0t = (float*)(ws + L.m0_t);
  int* flag = (int*)(ws + L.flag);
  float* dHs = (float*)(ws + L.dHs);
  float* dHt = (float*)(ws + L.dHt);
  const int64_t VC = P.vc;
  const int nt_max = (int)((VC + kStatTile - 1) / kStatTile);
  const bool two_pass = (algo >> 28) & 1;
  auto exp_first = VC <= 16384 ? exp_first_kernel<8> : exp_first_kernel<16>;
  // the two-pass combine over rows [r0, r0 + rg): one row per block, or (conditional
  // recomputation) a small grid walking the rows
  auto combine_soft = [&](int64_t rg, int64_t r0, int64_t vc, int nt, const float2* ss,
                          const float2* stt, __nv_bfloat16* Zs, __nv_bfloat16* Zt,
                          const int* run_if, cudaStream_t s) {
    const int64_t cap = 2 * (int64_t)sm_count();
    const unsigned grid = (unsigned)(run_if && rg > cap ? cap : rg);
    if (VC <= 16384)
      combine_soft_kernel<256><<<grid, 256, 0, s>>>(rg, vc, nt, nt_max, ss, stt, Zs, Zt, VC,
                                                    m + r0, l + r0, alpha + r0, mt + r0, lt + r0,
                                                    szt + r0, alpha_t + r0, run_if);
    else
      combine_soft_kernel<512><<<grid, 512, 0, s>>>(rg, vc, nt, nt_max, ss, stt, Zs, Zt, VC,
                                                    m + r0, l + r0, alpha + r0, mt + r0, lt + r0,
                                                    szt + r0, alpha_t + r0, run_if);
  };
  cudaStream_t side = side_stream(0);
  cudaEvent_t ev_fork = pool_event(0), ev_join = pool_event(1);
  cudaEvent_t ev_logits[2] = {pool_event(2), pool_event(3)};
  cudaEvent_t ev_dh[2] = {pool_event(4), pool_event(5)};
  if (!side || !ev_fork || !ev_join || !ev_logits[0] || !ev_logits[1] || !ev_dh[0] || !ev_dh[1]) {
    set_error("lmhead_ce: could not create the side stream or its events");
    return PE_ERR_CUDA;
  }
  soft_init_kernel<<<grid_for(R), 256, 0, st>>>(R, m, l, mt, lt, szt, ks_last, kt_last, flag,
                                                nullptr);
  PE_LAUNCHED();
  PE_CUDA_TRY(cudaEventRecord(ev_fork, st));
  PE_CUDA_TRY(cudaStreamWaitEvent(side, ev_fork, 0));
  int64_t t = 0;
  for (int64_t r0 = 0; r0 < R; r0 += P.rg) {
    const int64_t rg = (R - r0) < P.rg ? (R - r0) : P.rg;
    const void* hg = (const __nv_bfloat16*)h + r0 * ldh;
    const void* tg = (const __nv_bfloat16*)teacher + r0 * ldt;
    float* dHsg = dHs + r0 * H;
    float* dHtg = dHt + r0 * H;
    const unsigned fold_grid = (unsigned)((rg + 7) / 8);
    for (int64_t v0 = 0; v0 < V; v0 += VC, ++t) {
      const int b = (int)(t & 1);
      const int64_t vc = (V - v0) < VC ? (V - v0) : VC;
      const int nt = (int)((vc + kStatTile - 1) / kStatTile);
      const __nv_bfloat16* Wc = (const __nv_bfloat16*)W + v0 * H;
      __nv_bfloat16* Zs = (__nv_bfloat16*)(ws + L.Zs[b]);
      __nv_bfloat16* Zt = (__nv_bfloat16*)(ws + L.Zt[b]);
      float2* ss = (float2*)(ws + L.stats_s[b]);
      float2* stt = (float2*)(ws + L.stats_t[b]);
      float* kst = ks[t % 3] + r0;
      float* ktt = kt[t % 3] + r0;
      if (t >= 2) PE_CUDA_TRY(cudaStreamWaitEvent(st, ev_dh[b], 0));
      int rc;
      if (two_pass || v0 == 0) {
        rc = gemm_tc_logits_stats(rg, vc, H, hg, ldh, Wc, H, Zs, VC, ss, nt_max, status, st,
                                  P.logits_bn);
        if (!rc)
          rc = gemm_tc_logits_stats(rg, vc, H, tg, ldt, Wc, H, Zt, VC, stt, nt_max, status, st,
                                    P.logits_bn);
        if (rc) return rc;
        if (!two_pass) {
          fold_first_kernel<<<fold_grid, 256, 0, st>>>(rg, vc, nt, nt_max, ss, Zs, VC, nullptr,
                                                       m + r0, l + r0, m0s + r0, zlab + r0, kst,
                                                       ks_last + r0);
          PE_LAUNCHED();
          fold_first_kernel<<<fold_grid, 256, 0, st>>>(rg, vc, nt, nt_max, stt, Zt, VC, nullptr,
                                                       mt + r0, lt + r0, m0t + r0, zlab + r0,
                                                       ktt, kt_last + r0);
          PE_LAUNCHED();
        }
        PE_CUDA_TRY(cudaEventRecord(ev_logits[b], st));
        PE_CUDA_TRY(cudaStreamWaitEvent(side, ev_logits[b], 0));
        if (two_pass) {
          combine_soft(rg, r0, vc, nt, ss, stt, Zs, Zt, nullptr, side);
        } else {
          exp_first<<<(unsigned)rg, 256, 0, side>>>(vc, Zs, VC, nullptr, m0s + r0);
          PE_LAUNCHED();
          exp_first<<<(unsigned)rg, 256, 0, side>>>(vc, Zt, VC, nullptr, m0t + r0);
        }
        PE_LAUNCHED();
        // two-pass chunks rescale by the combine's alpha; a first chunk ignores the
        // factor (no accumulated input)
        rc = gemm_tc_rowscale_acc(rg, H, vc, Zs, VC, Wc, H, dHsg, H, v0 > 0 ? dHsg : nullptr,
                                  two_pass ? alpha + r0 : kst, status, side, P.dh_bn);
        if (!rc)
          rc = gemm_tc_rowscale_acc(rg, H, vc, Zt, VC, Wc, H, dHtg, H, v0 > 0 ? dHtg : nullptr,
                                    two_pass ? alpha_t + r0 : ktt, status, side, P.dh_bn);
      } else {
        rc = gemm_tc_logits_pexp(rg, vc, H, hg, ldh, Wc, H, Zs, VC, ss, nt_max, m + r0, nullptr,
                                 v0, nullptr, flag, status, st, P.logits_bn);
        if (!rc)
          rc = gemm_tc_logits_pexp(rg, vc, H, tg, ldt, Wc, H, Zt, VC, stt, nt_max, mt + r0,
                                   nullptr, v0, nullptr, flag, status, st, P.logits_bn);
        if (rc) return rc;
        fold_kernel<<<fold_grid, 256, 0, st>>>(rg, nt, nt_max, ss, m + r0, l + r0, kst,
                                               ks_last + r0);
        PE_LAUNCHED();
        fold_kernel<<<fold_grid, 256, 0, st>>>(rg, nt, nt_max, stt, mt + r0, lt + r0, ktt,
                                               kt_last + r0);
        PE_LAUNCHED();
        PE_CUDA_TRY(cudaEventRecord(ev_logits[b], st));
        PE_CUDA_TRY(cudaStreamWaitEvent(side, ev_logits[b], 0));
        rc = gemm_tc_rowscale_acc(rg, H, vc, Zs, VC, Wc, H, dHsg, H, dHsg, ks[(t + 2) % 3] + r0,
                                  status, side, P.dh_bn);
        if (!rc)
          rc = gemm_tc_rowscale_acc(rg, H, vc, Zt, VC, Wc, H, dHtg, H, dHtg,
                                    kt[(t + 2) % 3] + r0, status, side, P.dh_bn);
      }
      if (rc) return rc;
      PE_CUDA_TRY(cudaEventRecord(ev_dh[b], side));
    }
  }
  PE_CUDA_TRY(cudaEventRecord(ev_join, side));
  PE_CUDA_TRY(cudaStreamWaitEvent(st, ev_join, 0));
  if (!two_pass) {
    // S_tz from the teacher's dH (before a recomputation, which would overwrite it)
    soft_tz_kernel<<<(unsigned)((R + 7) / 8), 256, 0, st>>>(R, H, (const __nv_bfloat16*)h, ldh,
                                                            dHt, kt_last, szt);
    PE_LAUNCHED();
    // recomputation after an overflow: every launch conditional on the overflow word
    soft_init_kernel<<<grid_for(R), 256, 0, st>>>(R, m, l, mt, lt, szt, ks_last, kt_last,
                                                  nullptr, flag);
    PE_LAUNCHED();
    __nv_bfloat16* Zs = (__nv_bfloat16*)(ws + L.Zs[0]);
    __nv_bfloat16* Zt = (__nv_bfloat16*)(ws + L.Zt[0]);
    float2* ss = (float2*)(ws + L.stats_s[0]);
    float2* stt = (float2*)(ws + L.stats_t[0]);
    for (int64_t r0 = 0; r0 < R; r0 += P.rg) {
      const int64_t rg = (R - r0) < P.rg ? (R - r0) : P.rg;
      const void* hg = (const __nv_bfloat16*)h + r0 * ldh;
      const void* tg = (const __nv_bfloat16*)teacher + r0 * ldt;
      float* dHsg = dHs + r0 * H;
      float* dHtg = dHt + r0 * H;
      for (int64_t v0 = 0; v0 < V; v0 += VC) {
        const int64_t vc = (V - v0) < VC ? (V - v0) : VC;
        const int nt = (int)((vc + kStatTile - 1) / kStatTile);
        const __nv_bfloat16* Wc = (const __nv_bfloat16*)W + v0 * H;
        int rc = gemm_tc_logits_stats(rg, vc, H, hg, ldh, Wc, H, Zs, VC, ss, nt_max, status, st,
                                      P.logits_bn, flag);
        if (!rc)
          rc = gemm_tc_logits_stats(rg, vc, H, tg, ldt, Wc, H, Zt, VC, stt, nt_max, status, st,
                                    P.logits_bn, flag);
        if (rc) return rc;
        combine_soft(rg, r0, vc, nt, ss, stt, Zs, Zt, flag, st);
        PE_LAUNCHED();
        rc = gemm_tc_rowscale_acc(rg, H, vc, Zs, VC, Wc, H, dHsg, H, v0 > 0 ? dHsg : nullptr,
                                  alpha + r0, status, st, P.dh_bn, flag);
        if (!rc)
          rc = gemm_tc_rowscale_acc(rg, H, vc, Zt, VC, Wc, H, dHtg, H, v0 > 0 ? dHtg : nullptr,
                                    alpha_t + r0, status, st, P.dh_bn, flag);
        if (rc) return rc;
      }
    }
  }
  finalize_kernel<<<1, kFinThreads, 0, st>>>(R, nullptr, m, l, zlab, mt, lt, szt, lse, lse_t,
                                             loss_sum);
  PE_LAUNCHED();
  soft_dh_kernel<<<grid_for(R * H / 8), 256, 0, st>>>(R, H, dHs, dHt, l, lt, ks_last, kt_last,
                                                      grad_scale, (__nv_bfloat16*)dh, lddh);
  PE_LAUNCHED();
  return PE_OK;
}

}  // namespace
}  // namespace pe

using namespace pe;

extern "C" size_t pe_lmhead_ce_workspace(int dtype, int64_t R, int64_t H, int64_t V, int soft) {
  if (R <= 0 || H <= 0 || V <= 0) return 0;
  size_t bytes = layout_of(dtype, R, H, V, soft).total;
  if (dtype == PE_BF16) {
    const size_t f = soft ? soft_layout_of(R, H, V).total : fast_layout_of(R, H, V).total;
    if (f > bytes) bytes = f;
  }
  return bytes;
}

extern "C" int pe_lmhead_ce(int dtype, int64_t R, int64_t H, int64_t V, const void* h, int64_t ldh,
                            const void* W, const int64_t* labels, const void* teacher,
                            int64_t ldt, float grad_scale, void* dh, int64_t lddh,
                            float* loss_sum, void* workspace, size_t workspace_bytes, int algo,
                            int32_t* status, void* stream) {
  PE_CHECK_ARG(R >= 0 && H > 0 && V > 0 && ldh >= H && lddh >= H, "lmhead_ce: bad shape");
  PE_CHECK_ARG(labels || teacher, "lmhead_ce: needs labels or teacher rows");
  PE_CHECK_ARG(R <= (1ll << 31) - 1, "lmhead_ce: too many rows");
  if (R == 0) return PE_OK;
  const int soft = teacher != nullptr;
  cudaStream_t st = as_stream(stream);
  const int tuning = algo;  // chunk / row-group overrides of the fast path
  algo &= 0xff;
  if (fast_eligible(dtype, H, V, h, ldh, W, teacher, dh, lddh, algo)) {
    const size_t need = fast_layout_of(R, H, V).total;
    PE_CHECK_ARG(workspace && workspace_bytes >= need, "lmhead_ce: workspace of %zu bytes needed",
                 need);
    return lmhead_fast(R, H, V, h, ldh, W, labels, grad_scale, dh, lddh, loss_sum,
                       static_cast<uint8_t*>(workspace), tuning, status, st);
  }
  if (soft_fast_eligible(dtype, H, V, h, ldh, W, teacher, ldt, dh, lddh, algo)) {
    const size_t need = soft_layout_of(R, H, V).total;
    PE_CHECK_ARG(workspace && workspace_bytes >= need, "lmhead_ce: workspace of %zu bytes needed",
                 need);
    return lmhead_fast_soft(R, H, V, h, ldh, W, teacher, ldt, grad_scale, dh, lddh, loss_sum,
                            static_cast<uint8_t*>(workspace), tuning, status, st);
  }
  const Layout L = layout_of(dtype, R, H, V, soft);
  PE_CHECK_ARG(workspace && workspace_bytes >= L.total,
               "lmhead_ce: workspace of %zu bytes needed", L.total);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  float* m = (float*)(ws + L.m);
  float* l = (float*)(ws + L.l);
  float* zlab = (float*)(ws + L.zlab);
  float* lse = (float*)(ws + L.lse);
  float* mt = soft ? (float*)(ws + L.mt) : nullptr;
  float* lt = soft ? (float*)(ws + L.lt) : nullptr;
  float* szt = soft ? (float*)(ws + L.szt) : nullptr;
  float* lse_t = soft ? (float*)(ws + L.lse_t) : nullptr;
  float* Z = (float*)(ws + L.Z);
  float* Zt = soft ? (float*)(ws + L.Zt) : nullptr;
  void* G = ws + L.G;
  float* dH = (float*)(ws + L.dH);
  const int64_t VC = chunk_of(V);
  const size_t esz = dtype == PE_F32 ? 4 : 2;
  const int64_t* lab = soft ? nullptr : labels;

  init_stats_kernel<<<grid_for(R), 256, 0, st>>>(R, m, l, zlab, mt, lt, szt);
  PE_LAUNCHED();
  int rc;
  for (int64_t v0 = 0; v0 < V; v0 += VC) {
    const int64_t vc = (V - v0) < VC ? (V - v0) : VC;
    const void* Wc = (const uint8_t*)W + (size_t)v0 * H * esz;
    rc = gemm(dtype, R, vc, H, h, ldh, 1, Wc, H, 1, Z, VC, PE_F32, nullptr, 0, 1.f, 0.f, algo,
              status, st);
    if (rc) return rc;
    if (soft) {
      rc = gemm(dtype, R, vc, H, teacher, ldt, 1, Wc, H, 1, Zt, VC, PE_F32, nullptr, 0, 1.f, 0.f,
                algo, status, st);
      if (rc) return rc;
    }
    rc = PE_DISPATCH(dtype, T, [&] {
      stats_kernel<T><<<(unsigned)R, kThreads, 0, st>>>(vc, v0, Z, Zt, VC, lab, m, l, zlab, mt,
                                                        lt, szt);
      PE_LAUNCHED();
      return PE_OK;
    });
    if (rc) return rc;
  }
  finalize_kernel<<<1, kFinThreads, 0, st>>>(R, lab, m, l, zlab, mt, lt, szt, lse, lse_t, loss_sum);
  PE_LAUNCHED();
  for (int64_t v0 = 0; v0 < V; v0 += VC) {
    const int64_t vc = (V - v0) < VC ? (V - v0) : VC;
    const void* Wc = (const uint8_t*)W + (size_t)v0 * H * esz;
    rc = gemm(dtype, R, vc, H, h, ldh, 1, Wc, H, 1, Z, VC, PE_F32, nullptr, 0, 1.f, 0.f, algo,
              status, st);
    if (rc) return rc;
    if (soft) {
      rc = gemm(dtype, R, vc, H, teacher, ldt, 1, Wc, H, 1, Zt, VC, PE_F32, nullptr, 0, 1.f, 0.f,
                algo, status, st);
      if (rc) return rc;
    }
    rc = PE_DISPATCH(dtype, T, [&] {
      grad_kernel<T><<<grid_for(R * vc), 256, 0, st>>>(R, vc, v0, Z, Zt, VC, lab, lse, lse_t,
                                                       grad_scale, (T*)G, VC);
      PE_LAUNCHED();
      return PE_OK;
    });
    if (rc) return rc;
    // dH (+)= G[R, vc] * W_c[vc, H]   (W_c is the MN-major B operand)
    rc = gemm(dtype, R, H, vc, G, VC, 1, Wc, 1, H, dH, H, PE_F32, v0 > 0 ? dH : nullptr, H, 1.f,
              v0 > 0 ? 1.f : 0.f, algo, status, st);
    if (rc) return rc;
  }
  return PE_DISPATCH(dtype, T, [&] {
    cast2d_kernel<T><<<grid_for(R * H), 256, 0, st>>>(R, H, dH, (T*)dh, lddh);
    PE_LAUNCHED();
    return PE_OK;
  });
}
