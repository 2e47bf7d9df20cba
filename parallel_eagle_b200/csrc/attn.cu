// Attention entry points: argument checks and dispatch between the tensor-core
// kernels (bf16, head_dim 128, partition layout) and the CUDA-core kernels.
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
