// Attention entry points: argument checks and dispatch between the tensor-core
// kernels (bf16, head_dim 128, partition layout) and the CUDA-core kernels.
#include <vector>

#include "attn.cuh"

namespace pe {

static size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

static int check_common(int64_t B, int64_t S, int Hq, int Hkv, int hd, int layout, int64_t a0,
                        int64_t a1, int kd, const int32_t* anchor, const int32_t* depth,
                        const void* bias) {
  PE_CHECK_ARG(B >= 1 && S >= 0 && Hq >= 1 && Hkv >= 1 && hd >= 1, "attention: bad shape");
  PE_CHECK_ARG(Hq % Hkv == 0, "attention: n_heads %% n_kv_heads != 0");
  PE_CHECK_ARG(B <= 65535 && Hq <= 65535, "attention: grid limits");
  if (layout == PE_LAYOUT_PARTITION) {
    PE_CHECK_ARG(B == 1, "attention: partition layout is per sequence (B == 1)");
    PE_CHECK_ARG(kd >= 1 && 0 <= a0 && a0 < a1, "attention: bad partition (a0, a1, K)");
    PE_CHECK_ARG(S == a1 + (a1 - a0) * (kd - 1), "attention: S != a1 + (a1 - a0) * (K - 1)");
  } else if (layout == PE_LAYOUT_INDEXED) {
    PE_CHECK_ARG(anchor && depth, "attention: indexed layout needs anchor/depth");
  } else if (layout == PE_LAYOUT_BIAS) {
    PE_CHECK_ARG(bias != nullptr, "attention: bias layout needs a bias");
  } else {
    set_error("attention: unknown layout %d", layout);
    return PE_ERR_ARG;
  }
  return PE_OK;
}

}  // namespace pe

using namespace pe;

extern "C" int pe_attn_fwd(int dtype, int64_t B, int64_t S, int Hq, int Hkv, int head_dim,
                           const void* q, int64_t q_sb, int64_t q_ss, const void* k,
                           int64_t k_sb, int64_t k_ss, const void* v, int64_t v_sb,
                           int64_t v_ss, void* o, int64_t o_sb, int64_t o_ss, float* lse,
                           int layout, int64_t a0, int64_t a1, int kdepth,
                           const int32_t* anchor, const int32_t* depth, const void* bias,
                           int64_t bias_sb, int64_t bias_sq, int algo, int32_t* status,
                           void* stream) {
  int rc = check_common(B, S, Hq, Hkv, head_dim, layout, a0, a1, kdepth, anchor, depth, bias);
  if (rc) return rc;
  if (S == 0) return PE_OK;
  MaskSpec m{layout, a0, a1, kdepth, anchor, depth, bias, bias_sb, bias_sq};
  const bool tc = attn_tc_eligible(dtype, B, S, Hq, Hkv, head_dim, layout, q, q_ss, k, k_ss, v,
                                   v_ss);
  // algo bits 8-15: tensor-core kernel variant (0 two query tiles per CTA, 1 one)
  const int variant = (algo >> 8) & 0xff;
  algo &= 0xff;
  PE_CHECK_ARG(variant <= 1, "attention: unknown kernel variant %d", variant);
  if (algo == PE_ALGO_TCGEN05) PE_CHECK_ARG(tc, "attention: inputs not eligible for tcgen05");
  if (tc && algo != PE_ALGO_SIMT)
    return attn_fwd_tc_launch(S, Hq, Hkv, q, q_ss, k, k_ss, v, v_ss, o, o_ss, lse, m, status,
                              as_stream(stream), variant);
  return attn_fwd_simt_launch(dtype, B, S, Hq, Hkv, head_dim, q, q_sb, q_ss, k, k_sb, k_ss, v,
                              v_sb, v_ss, o, o_sb, o_ss, lse, m, as_stream(stream));
}

extern "C" int pe_attn_bwd(int dtype, int64_t B, int64_t S, int Hq, int Hkv, int head_dim,
                           const void* q, int64_t q_sb, int64_t q_ss, const void* k,
                           int64_t k_sb, int64_t k_ss, const void* v, int64_t v_sb,
                           int64_t v_ss, const void* o, int64_t o_sb, int64_t o_ss,
                           const void* dout, int64_t do_sb, int64_t do_ss, const float* lse,
                           void* dq, int64_t dq_sb, int64_t dq_ss, void* dk, int64_t dk_sb,
                           int64_t dk_ss, void* dv, int64_t dv_sb, int64_t dv_ss,
                           void* workspace, size_t workspace_bytes, int layout, int64_t a0,
                           int64_t a1, int kdepth, const int32_t* anchor, const int32_t* depth,
                           const void* bias, int64_t bias_sb, int64_t bias_sq, int algo,
                           int32_t* status, void* stream) {
  int rc = check_common(B, S, Hq, Hkv, head_dim, layout, a0, a1, kdepth, anchor, depth, bias);
  if (rc) return rc;
  if (S == 0) return PE_OK;
  const size_t delta_bytes = align256((size_t)B * Hq * S * 4);
  PE_CHECK_ARG(workspace && workspace_bytes >= delta_bytes,
               "attention backward: workspace too small (see pe_attn_bwd_workspace)");
  float* delta = static_cast<float*>(workspace);
  MaskSpec m{layout, a0, a1, kdepth, anchor, depth, bias, bias_sb, bias_sq};
  // algo bits 8-15: tensor-core kernel variant (0 dQ kernel + persistent dK-dV kernel,
  // 1 fused kernel with dQ atomics, 2 dQ kernel + one-CTA-per-tile dK-dV kernel)
  const int variant = (algo >> 8) & 0xff;
  algo &= 0xff;
  PE_CHECK_ARG(variant <= 2, "attention backward: unknown kernel variant %d", variant);
  const bool tc = attn_tc_bwd_ready() &&
                  attn_tc_eligible(dtype, B, S, Hq, Hkv, head_dim, layout, q, q_ss, k, k_ss, v,
                                   v_ss) &&
                  workspace_bytes >= delta_bytes + attn_tc_bwd_acc_bytes(S, Hq, Hkv);
  if (algo == PE_ALGO_TCGEN05) PE_CHECK_ARG(tc, "attention: inputs not eligible for tcgen05");
  if (tc && algo != PE_ALGO_SIMT) {
    float* dq_acc = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + delta_bytes);
    return attn_bwd_tc_launch(S, Hq, Hkv, q, q_ss, k, k_ss, v, v_ss, o, o_ss, dout, do_ss, lse,
                              dq, dq_ss, dk, dk_ss, dv, dv_ss, delta, dq_acc, m, status,
                              as_stream(stream), variant);
  }
  return attn_bwd_simt_launch(dtype, B, S, Hq, Hkv, head_dim, q, q_sb, q_ss, k, k_sb, k_ss, v,
                              v_sb, v_ss, o, o_sb, o_ss, dout, do_sb, do_ss, lse, dq, dq_sb,
                              dq_ss, dk, dk_sb, dk_ss, dv, dv_sb, dv_ss, delta, m,
                              as_stream(stream));
}

extern "C" size_t pe_attn_bwd_workspace(int dtype, int64_t B, int64_t S, int Hq, int Hkv,
                                        int head_dim) {
  if (B <= 0 || S <= 0 || Hq <= 0 || Hkv <= 0 || head_dim <= 0) return 0;
  size_t bytes = align256((size_t)B * Hq * S * 4);
  if (dtype == PE_BF16 && B == 1 && head_dim == 128)
    bytes += align256(attn_tc_bwd_acc_bytes(S, Hq, Hkv));
  return bytes;
}

// ------------------------------------------------------ stacked segments ----

namespace pe {

// geometry of the stacked segments; false (with the error set) on a bad table
static bool seg_geoms(int nseg, const int64_t* bounds, int kdepth,
                      std::vector<attn_tc::PartGeom>& g, int64_t& rows) {
  if (nseg < 1 || !bounds || kdepth < 1) {
    set_error("attention segments: need nseg >= 1, bounds and kdepth >= 1");
    return false;
  }
  g.resize(nseg);
  rows = 0;
  for (int s = 0; s < nseg; ++s) {
    const int64_t a0 = bounds[2 * s], a1 = bounds[2 * s + 1];
    const int64_t S = a1 + (a1 - a0) * (kdepth - 1);
    if (!(0 <= a0 && a0 < a1) || S > 65535ll * 128) {
      set_error("attention segments: bad segment %d (a0 %lld, a1 %lld)", s, (long long)a0,
                (long long)a1);
      return false;
    }
    g[s] = attn_tc::PartGeom{(int)S, (int)a0, (int)a1, kdepth - 1};
    rows += S;
  }
  return true;
}

static size_t elem_bytes(int dtype) { return dtype == PE_F32 ? 4 : 2; }

static size_t seg_workspace(int dtype, int64_t rows, int Hq, int Hkv, int head_dim) {
  size_t bytes = align256((size_t)Hq * rows * 4);  // deltas
  if (dtype == PE_BF16 && head_dim == 128) bytes += align256(attn_tc_seg_acc_bytes(rows, Hkv));
  return bytes;
}

}  // namespace pe

extern "C" int pe_attn_fwd_segments(int dtype, int nseg, const int64_t* bounds, int kdepth,
                                    int Hq, int Hkv, int head_dim, const void* q, int64_t q_ss,
                                    const void* k, int64_t k_ss, const void* v, int64_t v_ss,
                                    void* o, int64_t o_ss, float* lse, int algo,
                                    int32_t* status, void* stream) {
  std::vector<attn_tc::PartGeom> g;
  int64_t rows = 0;
  if (!seg_geoms(nseg, bounds, kdepth, g, rows)) return PE_ERR_ARG;
  PE_CHECK_ARG(Hq >= 1 && Hkv >= 1 && head_dim >= 1 && Hq % Hkv == 0 && Hq <= 65535,
               "attention segments: bad head counts");
  // bits 16-19: the forward's exponential-emulation ratio + 1 (0: default); no other
  // variant bits
  PE_CHECK_ARG(((algo >> 8) & ~0xf00) == 0,
               "attention segments: kernel-variant bits other than the forward's "
               "exp-emulation bits 16-19 are not accepted");
  const int emu = ((algo >> 16) & 0xf) - 1;
  algo &= 0xff;
  bool tc = true;
  for (int s = 0; s < nseg; ++s)
    tc = tc && attn_tc_eligible(dtype, 1, g[s].S, Hq, Hkv, head_dim, PE_LAYOUT_PARTITION, q, q_ss,
                                k, k_ss, v, v_ss);
  if (algo == PE_ALGO_TCGEN05) PE_CHECK_ARG(tc, "attention: inputs not eligible for tcgen05");
  if (tc && algo != PE_ALGO_SIMT)
    return attn_fwd_tc_segments(nseg, g.data(), Hq, Hkv, q, q_ss, k, k_ss, v, v_ss, o, o_ss, lse,
                                status, as_stream(stream), emu);
  PE_CHECK_ARG(dtype == PE_F32 || dtype == PE_BF16, "attention segments: unknown dtype %d", dtype);
  const size_t es = elem_bytes(dtype);
  int64_t row0 = 0;
  for (int s = 0; s < nseg; ++s) {
    const int64_t S = g[s].S;
    MaskSpec m{PE_LAYOUT_PARTITION, g[s].a0, g[s].a1, kdepth, nullptr, nullptr, nullptr, 0, 0};
    const int rc = attn_fwd_simt_launch(
        dtype, 1, S, Hq, Hkv, head_dim, static_cast<const uint8_t*>(q) + row0 * q_ss * es, 0,
        q_ss, static_cast<const uint8_t*>(k) + row0 * k_ss * es, 0, k_ss,
        static_cast<const uint8_t*>(v) + row0 * v_ss * es, 0, v_ss,
        static_cast<uint8_t*>(o) + row0 * o_ss * es, 0, o_ss, lse + Hq * row0, m,
        as_stream(stream));
    if (rc) return rc;
    row0 += S;
  }
  return PE_OK;
}

extern "C" size_t pe_attn_bwd_segments_workspace(int dtype, int nseg, const int64_t* bounds,
                                                 int kdepth, int Hq, int Hkv, int head_dim) {
  std::vector<attn_tc::PartGeom> g;
  int64_t rows = 0;
  if (Hq <= 0 || Hkv <= 0 || head_dim <= 0 || !seg_geoms(nseg, bounds, kdepth, g, rows)) return 0;
  return seg_workspace(dtype, rows, Hq, Hkv, head_dim);
}

extern "C" int pe_attn_bwd_segments(int dtype, int nseg, const int64_t* bounds, int kdepth,
                                    int Hq, int Hkv, int head_dim, const void* q, int64_t q_ss,
                                    const void* k, int64_t k_ss, const void* v, int64_t v_ss,
                                    const void* o, int64_t o_ss, const void* dout,
                                    int64_t do_ss, const float* lse, void* dq, int64_t dq_ss,
                                    void* dk, int64_t dk_ss, void* dv, int64_t dv_ss,
                                    void* workspace, size_t workspace_bytes,
                                    const void* rope_cs, int64_t cs_ld, int algo,
                                    int32_t* status, void* stream) {
  std::vector<attn_tc::PartGeom> g;
  int64_t rows = 0;
  if (!seg_geoms(nseg, bounds, kdepth, g, rows)) return PE_ERR_ARG;
  PE_CHECK_ARG(Hq >= 1 && Hkv >= 1 && head_dim >= 1 && Hq % Hkv == 0 && Hq <= 65535,
               "attention segments: bad head counts");
  PE_CHECK_ARG((algo >> 8) == 0, "attention segments: kernel-variant bits are not accepted");
  const size_t delta_bytes = align256((size_t)Hq * rows * 4);
  PE_CHECK_ARG(workspace && workspace_bytes >= delta_bytes,
               "attention backward: workspace too small (see pe_attn_bwd_segments_workspace)");
  float* delta = static_cast<float*>(workspace);
  bool tc = attn_tc_bwd_ready() &&
            workspace_bytes >= delta_bytes + attn_tc_seg_acc_bytes(rows, Hkv);
  for (int s = 0; s < nseg; ++s)
    tc = tc && attn_tc_eligible(dtype, 1, g[s].S, Hq, Hkv, head_dim, PE_LAYOUT_PARTITION, q, q_ss,
                                k, k_ss, v, v_ss);
  if (algo == PE_ALGO_TCGEN05) PE_CHECK_ARG(tc, "attention: inputs not eligible for tcgen05");
  if (tc && algo != PE_ALGO_SIMT) {
    float* acc = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + delta_bytes);
    return attn_bwd_tc_segments(nseg, g.data(), Hq, Hkv, q, q_ss, k, k_ss, v, v_ss, o, o_ss, dout,
                                do_ss, lse, dq, dq_ss, dk, dk_ss, dv, dv_ss, delta, acc, rope_cs,
                                cs_ld, status, as_stream(stream));
  }
  PE_CHECK_ARG(!rope_cs || cs_ld >= head_dim, "attention segments: rotary table rows too short");
  PE_CHECK_ARG(dtype == PE_F32 || dtype == PE_BF16, "attention segments: unknown dtype %d", dtype);
  const size_t es = elem_bytes(dtype);
  auto at = [es](const void* p, int64_t row, int64_t ss) {
    return static_cast<const uint8_t*>(p) + row * ss * es;
  };
  auto at_mut = [es](void* p, int64_t row, int64_t ss) {
    return static_cast<uint8_t*>(p) + row * ss * es;
  };
  int64_t row0 = 0;
  for (int s = 0; s < nseg; ++s) {
    const int64_t S = g[s].S;
    MaskSpec m{PE_LAYOUT_PARTITION, g[s].a0, g[s].a1, kdepth, nullptr, nullptr, nullptr, 0, 0};
    const int rc = attn_bwd_simt_launch(
        dtype, 1, S, Hq, Hkv, head_dim, at(q, row0, q_ss), 0, q_ss, at(k, row0, k_ss), 0, k_ss,
        at(v, row0, v_ss), 0, v_ss, at(o, row0, o_ss), 0, o_ss, at(dout, row0, do_ss), 0, do_ss,
        lse + Hq * row0, at_mut(dq, row0, dq_ss), 0, dq_ss, at_mut(dk, row0, dk_ss), 0, dk_ss,
        at_mut(dv, row0, dv_ss), 0, dv_ss, delta + Hq * row0, m, as_stream(stream));
    if (rc) return rc;
    row0 += S;
  }
  if (rope_cs) {
    // CUDA-core path: the same inverse rotation as a separate pass over dq and dk
    int rc = rope_apply_table(dtype, rows, Hq, head_dim, dq, dq_ss, rope_cs, cs_ld, 1,
                              as_stream(stream));
    if (!rc)
      rc = rope_apply_table(dtype, rows, Hkv, head_dim, dk, dk_ss, rope_cs, cs_ld, 1,
                            as_stream(stream));
    if (rc) return rc;
  }
  return PE_OK;
}
