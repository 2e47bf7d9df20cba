// CUDA-core cross-depth masked attention (forward and backward), fp32 math.
//
// The fp32-mode path and the reference implementation the tensor-core kernels
// are tested against.  One warp per query (or, for dK/dV, per key) row; lanes
// split the head dimension.  The attend rule is re-derived per pair, and in the
// partition layout the kernel visits only the slots the rule allows: a query
// (i, d) reads the real keys 0..i and its own anchor's prediction keys
// 1..d; a real key j is read by the real queries j..a1-1 and by every prediction
// slot of anchors >= j.  Online softmax in fp32.
#include "attn.cuh"

namespace pe {
namespace {

constexpr int kMaxDPL = 4;  // head_dim <= 128
constexpr int kWarps = 4;

struct Range {
  int64_t lo, hi;
};

// key ranges visited by query slot s; check=true means "test every pair"
__device__ __forceinline__ int query_ranges(const MaskSpec& m, int64_t S, int64_t s, Range* r,
                                            bool& check) {
  if (m.layout == PE_LAYOUT_PARTITION) {
    check = false;
    int64_t i;
    int d;
    slot_decode(m, s, i, d);
    r[0] = {0, i + 1};
    if (d >= 1) {
      const int64_t base = m.a1 + (i - m.a0) * (m.kd - 1);
      r[1] = {base, base + d};
      return 2;
    }
    return 1;
  }
  check = m.layout == PE_LAYOUT_INDEXED;
  r[0] = {0, S};
  return 1;
}

// query ranges that read key slot j
__device__ __forceinline__ int key_ranges(const MaskSpec& m, int64_t S, int64_t j, Range* r,
                                          bool& check) {
  if (m.layout == PE_LAYOUT_PARTITION) {
    check = false;
    int64_t a;
    int e;
    slot_decode(m, j, a, e);
    if (e == 0) {
      r[0] = {a, m.a1};
      const int64_t first = a > m.a0 ? a : m.a0;
      r[1] = {m.a1 + (first - m.a0) * (m.kd - 1), S};
      return 2;
    }
    const int64_t base = m.a1 + (a - m.a0) * (m.kd - 1);
    r[0] = {base + (e - 1), base + (m.kd - 1)};
    return 1;
  }
  check = m.layout == PE_LAYOUT_INDEXED;
  r[0] = {0, S};
  return 1;
}

template <typename T>
__device__ __forceinline__ void load_row(const T* p, int hd, int lane, float* v) {
#pragma unroll
  for (int t = 0; t < kMaxDPL; ++t) {
    const int d = lane + 32 * t;
    v[t] = d < hd ? to_f(p[d]) : 0.f;
  }
}

__device__ __forceinline__ float dot_row(const float* a, const float* b) {
  float s = 0.f;
#pragma unroll
  for (int t = 0; t < kMaxDPL; ++t) s += a[t] * b[t];
  return warp_sum(s);
}

template <typename T>
__device__ __forceinline__ float bias_at(const MaskSpec& m, int64_t b, int64_t s, int64_t j) {
  const T* bp = reinterpret_cast<const T*>(m.bias);
  return to_f(bp[b * m.bias_sb + s * m.bias_sq + j]);
}

template <typename T>
__global__ void __launch_bounds__(kWarps * 32)
attn_fwd_simt(int64_t S, int Hq, int Hkv, int hd, const T* q, int64_t q_sb, int64_t q_ss,
              const T* k, int64_t k_sb, int64_t k_ss, const T* v, int64_t v_sb, int64_t v_ss,
              T* o, int64_t o_sb, int64_t o_ss, float* lse, MaskSpec m, float scale) {
  const int lane = threadIdx.x & 31;
  const int64_t s = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  const int h = blockIdx.y;
  const int64_t b = blockIdx.z;
  if (s >= S) return;
  const int kvh = h / (Hq / Hkv);
  float qv[kMaxDPL];
  load_row(q + b * q_sb + s * q_ss + (int64_t)h * hd, hd, lane, qv);
  int64_t qi = 0;
  int qd = 0;
  if (m.layout == PE_LAYOUT_INDEXED) slot_decode(m, s, qi, qd);
  Range rg[2];
  bool check;
  const int nr = query_ranges(m, S, s, rg, check);
  float mx = -INFINITY, l = 0.f, acc[kMaxDPL] = {0.f, 0.f, 0.f, 0.f};
  for (int ri = 0; ri < nr; ++ri) {
    for (int64_t j = rg[ri].lo; j < rg[ri].hi; ++j) {
      if (check) {
        int64_t kj;
        int kdp;
        slot_decode(m, j, kj, kdp);
        if (!mtp_allowed(qi, qd, kj, kdp)) continue;
      }
      float kv[kMaxDPL];
      load_row(k + b * k_sb + j * k_ss + (int64_t)kvh * hd, hd, lane, kv);
      float sc = dot_row(qv, kv) * scale;
      if (m.layout == PE_LAYOUT_BIAS) sc += bias_at<T>(m, b, s, j);
      const float mn = fmaxf(mx, sc);
      const float corr = expf(mx - mn);
      const float p = expf(sc - mn);
      float vv[kMaxDPL];
      load_row(v + b * v_sb + j * v_ss + (int64_t)kvh * hd, hd, lane, vv);
      l = l * corr + p;
#pragma unroll
      for (int t = 0; t < kMaxDPL; ++t) acc[t] = acc[t] * corr + p * vv[t];
      mx = mn;
    }
  }
  const float inv = 1.f / l;
  T* orow = o + b * o_sb + s * o_ss + (int64_t)h * hd;
#pragma unroll
  for (int t = 0; t < kMaxDPL; ++t) {
    const int d = lane + 32 * t;
    if (d < hd) orow[d] = from_f<T>(acc[t] * inv);
  }
  if (lane == 0) lse[(b * Hq + h) * S + s] = mx + logf(l);
}

// delta[b,h,s] = sum_d dO * O
template <typename T>
__global__ void attn_delta_simt(int64_t S, int Hq, int hd, const T* o, int64_t o_sb, int64_t o_ss,
                                const T* dout, int64_t do_sb, int64_t do_ss, float* delta) {
  const int lane = threadIdx.x & 31;
  const int64_t s = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  const int h = blockIdx.y;
  const int64_t b = blockIdx.z;
  if (s >= S) return;
  float a[kMaxDPL], c[kMaxDPL];
  load_row(o + b * o_sb + s * o_ss + (int64_t)h * hd, hd, lane, a);
  load_row(dout + b * do_sb + s * do_ss + (int64_t)h * hd, hd, lane, c);
  const float d = dot_row(a, c);
  if (lane == 0) delta[(b * Hq + h) * S + s] = d;
}

template <typename T>
__global__ void __launch_bounds__(kWarps * 32)
attn_dq_simt(int64_t S, int Hq, int Hkv, int hd, const T* q, int64_t q_sb, int64_t q_ss,
             const T* k, int64_t k_sb, int64_t k_ss, const T* v, int64_t v_sb, int64_t v_ss,
             const T* dout, int64_t do_sb, int64_t do_ss, const float* lse, const float* delta,
             T* dq, int64_t dq_sb, int64_t dq_ss, MaskSpec m, float scale) {
  const int lane = threadIdx.x & 31;
  const int64_t s = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  const int h = blockIdx.y;
  const int64_t b = blockIdx.z;
  if (s >= S) return;
  const int kvh = h / (Hq / Hkv);
  float qv[kMaxDPL], dov[kMaxDPL];
  load_row(q + b * q_sb + s * q_ss + (int64_t)h * hd, hd, lane, qv);
  load_row(dout + b * do_sb + s * do_ss + (int64_t)h * hd, hd, lane, dov);
  const float L = lse[(b * Hq + h) * S + s];
  const float D = delta[(b * Hq + h) * S + s];
  int64_t qi = 0;
  int qd = 0;
  if (m.layout == PE_LAYOUT_INDEXED) slot_decode(m, s, qi, qd);
  Range rg[2];
  bool check;
  const int nr = query_ranges(m, S, s, rg, check);
  float acc[kMaxDPL] = {0.f, 0.f, 0.f, 0.f};
  for (int ri = 0; ri < nr; ++ri) {
    for (int64_t j = rg[ri].lo; j < rg[ri].hi; ++j) {
      if (check) {
        int64_t kj;
        int kdp;
        slot_decode(m, j, kj, kdp);
        if (!mtp_allowed(qi, qd, kj, kdp)) continue;
      }
      float kv[kMaxDPL], vv[kMaxDPL];
      load_row(k + b * k_sb + j * k_ss + (int64_t)kvh * hd, hd, lane, kv);
      load_row(v + b * v_sb + j * v_ss + (int64_t)kvh * hd, hd, lane, vv);
      float sc = dot_row(qv, kv) * scale;
      if (m.layout == PE_LAYOUT_BIAS) sc += bias_at<T>(m, b, s, j);
      const float p = expf(sc - L);
      const float dp = dot_row(dov, vv);
      const float ds = p * (dp - D) * scale;
#pragma unroll
      for (int t = 0; t < kMaxDPL; ++t) acc[t] += ds * kv[t];
    }
  }
  T* row = dq + b * dq_sb + s * dq_ss + (int64_t)h * hd;
#pragma unroll
  for (int t = 0; t < kMaxDPL; ++t) {
    const int d = lane + 32 * t;
    if (d < hd) row[d] = from_f<T>(acc[t]);
  }
}

template <typename T>
__global__ void __launch_bounds__(kWarps * 32)
attn_dkdv_simt(int64_t S, int Hq, int Hkv, int hd, const T* q, int64_t q_sb, int64_t q_ss,
               const T* k, int64_t k_sb, int64_t k_ss, const T* v, int64_t v_sb, int64_t v_ss,
               const T* dout, int64_t do_sb, int64_t do_ss, const float* lse,
               const float* delta, T* dk, int64_t dk_sb, int64_t dk_ss, T* dv, int64_t dv_sb,
               int64_t dv_ss, MaskSpec m, float scale) {
  const int lane = threadIdx.x & 31;
  const int64_t j = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  const int kvh = blockIdx.y;
  const int64_t b = blockIdx.z;
  if (j >= S) return;
  const int rep = Hq / Hkv;
  float kv[kMaxDPL], vv[kMaxDPL];
  load_row(k + b * k_sb + j * k_ss + (int64_t)kvh * hd, hd, lane, kv);
  load_row(v + b * v_sb + j * v_ss + (int64_t)kvh * hd, hd, lane, vv);
  int64_t kj = 0;
  int kdp = 0;
  if (m.layout == PE_LAYOUT_INDEXED) slot_decode(m, j, kj, kdp);
  Range rg[2];
  bool check;
  const int nr = key_ranges(m, S, j, rg, check);
  float dka[kMaxDPL] = {0.f, 0.f, 0.f, 0.f}, dva[kMaxDPL] = {0.f, 0.f, 0.f, 0.f};
  for (int g = 0; g < rep; ++g) {
    const int h = kvh * rep + g;
    for (int ri = 0; ri < nr; ++ri) {
      for (int64_t s = rg[ri].lo; s < rg[ri].hi; ++s) {
        if (check) {
          int64_t qi;
          int qd;
          slot_decode(m, s, qi, qd);
          if (!mtp_allowed(qi, qd, kj, kdp)) continue;
        }
        float qv[kMaxDPL], dov[kMaxDPL];
        load_row(q + b * q_sb + s * q_ss + (int64_t)h * hd, hd, lane, qv);
        load_row(dout + b * do_sb + s * do_ss + (int64_t)h * hd, hd, lane, dov);
        float sc = dot_row(qv, kv) * scale;
        if (m.layout == PE_LAYOUT_BIAS) sc += bias_at<T>(m, b, s, j);
        const float p = expf(sc - lse[(b * Hq + h) * S + s]);
        const float dp = dot_row(dov, vv);
        const float ds = p * (dp - delta[(b * Hq + h) * S + s]) * scale;
#pragma unroll
        for (int t = 0; t < kMaxDPL; ++t) {
          dva[t] += p * dov[t];
          dka[t] += ds * qv[t];
        }
      }
    }
  }
  T* krow = dk + b * dk_sb + j * dk_ss + (int64_t)kvh * hd;
  T* vrow = dv + b * dv_sb + j * dv_ss + (int64_t)kvh * hd;
#pragma unroll
  for (int t = 0; t < kMaxDPL; ++t) {
    const int d = lane + 32 * t;
    if (d < hd) {
      krow[d] = from_f<T>(dka[t]);
      vrow[d] = from_f<T>(dva[t]);
    }
  }
}

}  // namespace

int attn_fwd_simt_launch(int dtype, int64_t B, int64_t S, int Hq, int Hkv, int hd,
                         const void* q, int64_t q_sb, int64_t q_ss, const void* k, int64_t k_sb,
                         int64_t k_ss, const void* v, int64_t v_sb, int64_t v_ss, void* o,
                         int64_t o_sb, int64_t o_ss, float* lse, const MaskSpec& m,
                         cudaStream_t st) {
  PE_CHECK_ARG(hd <= 32 * kMaxDPL, "attention (simt): head_dim > 128");
  const float scale = 1.0f / sqrtf((float)hd);
  dim3 grid((unsigned)ceil_div(S, kWarps), (unsigned)Hq, (unsigned)B);
  return PE_DISPATCH(dtype, T, [&] {
    attn_fwd_simt<T><<<grid, kWarps * 32, 0, st>>>(S, Hq, Hkv, hd, (const T*)q, q_sb, q_ss,
                                                   (const T*)k, k_sb, k_ss, (const T*)v, v_sb,
                                                   v_ss, (T*)o, o_sb, o_ss, lse, m, scale);
    PE_LAUNCHED();
    return PE_OK;
  });
}

int attn_bwd_simt_launch(int dtype, int64_t B, int64_t S, int Hq, int Hkv, int hd,
                         const void* q, int64_t q_sb, int64_t q_ss, const void* k, int64_t k_sb,
                         int64_t k_ss, const void* v, int64_t v_sb, int64_t v_ss, const void* o,
                         int64_t o_sb, int64_t o_ss, const void* dout, int64_t do_sb,
                         int64_t do_ss, const float* lse, void* dq, int64_t dq_sb, int64_t dq_ss,
                         void* dk, int64_t dk_sb, int64_t dk_ss, void* dv, int64_t dv_sb,
                         int64_t dv_ss, float* delta, const MaskSpec& m, cudaStream_t st) {
  PE_CHECK_ARG(hd <= 32 * kMaxDPL, "attention (simt): head_dim > 128");
  const float scale = 1.0f / sqrtf((float)hd);
  dim3 gq((unsigned)ceil_div(S, kWarps), (unsigned)Hq, (unsigned)B);
  dim3 gk((unsigned)ceil_div(S, kWarps), (unsigned)Hkv, (unsigned)B);
  return PE_DISPATCH(dtype, T, [&] {
    attn_delta_simt<T><<<gq, kWarps * 32, 0, st>>>(S, Hq, hd, (const T*)o, o_sb, o_ss,
                                                   (const T*)dout, do_sb, do_ss, delta);
    PE_LAUNCHED();
    attn_dq_simt<T><<<gq, kWarps * 32, 0, st>>>(
        S, Hq, Hkv, hd, (const T*)q, q_sb, q_ss, (const T*)k, k_sb, k_ss, (const T*)v, v_sb,
        v_ss, (const T*)dout, do_sb, do_ss, lse, delta, (T*)dq, dq_sb, dq_ss, m, scale);
    PE_LAUNCHED();
    attn_dkdv_simt<T><<<gk, kWarps * 32, 0, st>>>(
        S, Hq, Hkv, hd, (const T*)q, q_sb, q_ss, (const T*)k, k_sb, k_ss, (const T*)v, v_sb,
        v_ss, (const T*)dout, do_sb, do_ss, lse, delta, (T*)dk, dk_sb, dk_ss, (T*)dv, dv_sb,
        dv_ss, m, scale);
    PE_LAUNCHED();
    return PE_OK;
  });
}

}  // namespace pe
