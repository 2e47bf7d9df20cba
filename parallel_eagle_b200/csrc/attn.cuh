// Attend-rule reconstruction shared by the attention kernels.
//
// The MTP rule (reference src/pe/masks.py:43-61): query slot (i, d) sees key
// slot (j, e) iff  e == 0 ? j <= i : (j == i && e <= d).  In the partition
// layout (reference src/pe/partition.py:41-55) slot s < a1 is (s, 0) and slot
// a1 + t is (a0 + t / (K-1), 1 + t % (K-1)), so nothing but (a0, a1, K) is
// needed to know which pairs exist.
#pragma once
#include "common.cuh"

namespace pe {

namespace attn_tc {
// one segment of the partition layout: S = a1 + (a1 - a0) * km1 slots
struct PartGeom {
  int S, a0, a1, km1;  // km1 = K - 1 (0 when K == 1)
};
}  // namespace attn_tc

struct MaskSpec {
  int layout;
  int64_t a0, a1;
  int kd;
  const int32_t* anchor;
  const int32_t* depth;
  const void* bias;
  int64_t bias_sb, bias_sq;
};

__device__ __forceinline__ void slot_decode(const MaskSpec& m, int64_t s, int64_t& anc, int& dep) {
  if (m.layout == PE_LAYOUT_PARTITION) {
    if (s < m.a1) {
      anc = s;
      dep = 0;
    } else {
      const int64_t t = s - m.a1;
      const int per = m.kd - 1;
      anc = m.a0 + t / per;
      dep = 1 + (int)(t % per);
    }
  } else {
    anc = m.anchor[s];
    dep = m.depth[s];
  }
}

__device__ __forceinline__ bool mtp_allowed(int64_t ai, int di, int64_t aj, int dj) {
  return dj == 0 ? (aj <= ai) : (aj == ai && dj <= di);
}

int attn_fwd_simt_launch(int dtype, int64_t B, int64_t S, int Hq, int Hkv, int hd,
                         const void* q, int64_t q_sb, int64_t q_ss, const void* k, int64_t k_sb,
                         int64_t k_ss, const void* v, int64_t v_sb, int64_t v_ss, void* o,
                         int64_t o_sb, int64_t o_ss, float* lse, const MaskSpec& m,
                         cudaStream_t st);
int attn_bwd_simt_launch(int dtype, int64_t B, int64_t S, int Hq, int Hkv, int hd,
                         const void* q, int64_t q_sb, int64_t q_ss, const void* k, int64_t k_sb,
                         int64_t k_ss, const void* v, int64_t v_sb, int64_t v_ss, const void* o,
                         int64_t o_sb, int64_t o_ss, const void* dout, int64_t do_sb,
                         int64_t do_ss, const float* lse, void* dq, int64_t dq_sb, int64_t dq_ss,
                         void* dk, int64_t dk_sb, int64_t dk_ss, void* dv, int64_t dv_sb,
                         int64_t dv_ss, float* delta, const MaskSpec& m, cudaStream_t st);
bool attn_tc_eligible(int dtype, int64_t B, int64_t S, int Hq, int Hkv, int hd, int layout,
                      const void* q, int64_t q_ss, const void* k, int64_t k_ss, const void* v,
                      int64_t v_ss);
bool attn_tc_bwd_ready();
// fp32 dQ / dK / dV accumulators of the tensor-core backward
size_t attn_tc_bwd_acc_bytes(int64_t S, int Hq, int Hkv);
int attn_fwd_tc_launch(int64_t S, int Hq, int Hkv, const void* q, int64_t q_ss, const void* k,
                       int64_t k_ss, const void* v, int64_t v_ss, void* o, int64_t o_ss,
                       float* lse, const MaskSpec& m, int* status, cudaStream_t st,
                       int variant = 0);
int attn_bwd_tc_launch(int64_t S, int Hq, int Hkv, const void* q, int64_t q_ss, const void* k,
                       int64_t k_ss, const void* v, int64_t v_ss, const void* o, int64_t o_ss,
                       const void* dout, int64_t do_ss, const float* lse, void* dq,
                       int64_t dq_ss, void* dk, int64_t dk_ss, void* dv, int64_t dv_ss,
                       float* delta, float* dq_acc, const MaskSpec& m, int* status,
                       cudaStream_t st, int variant = 0);
// Stacked segments (tensor cores): segment s occupies rows [row0_s, row0_s + g[s].S)
// of every row operand, row0_0 = 0 and row0_{s+1} = row0_s + g[s].S; lse / delta hold
// one [Hq, g[s].S] block per segment starting at element Hq * row0_s.
// emu: one exponential pair in `emu` from the FMA-pipe polynomial (0: none; -1: the
// default ratio)
int attn_fwd_tc_segments(int nseg, const attn_tc::PartGeom* g, int Hq, int Hkv, const void* q,
                         int64_t q_ss, const void* k, int64_t k_ss, const void* v, int64_t v_ss,
                         void* o, int64_t o_ss, float* lse, int* status, cudaStream_t st,
                         int emu = -1);
// acc: fp32 dK / dV accumulators and the work counter, attn_tc_seg_acc_bytes(rows)
size_t attn_tc_seg_acc_bytes(int64_t rows, int Hkv);
// rope_cs (may be NULL): per stacked row [cos hd/2 | sin hd/2] table (row stride
// cs_ld); with it dq and dk leave rotated back by the transpose of the rotary
// embedding (gradients with respect to the unrotated q / k)
int attn_bwd_tc_segments(int nseg, const attn_tc::PartGeom* g, int Hq, int Hkv, const void* q,
                         int64_t q_ss, const void* k, int64_t k_ss, const void* v, int64_t v_ss,
                         const void* o, int64_t o_ss, const void* dout, int64_t do_ss,
                         const float* lse, void* dq, int64_t dq_ss, void* dk, int64_t dk_ss,
                         void* dv, int64_t dv_ss, float* delta, float* acc,
                         const void* rope_cs, int64_t cs_ld, int* status, cudaStream_t st);
// x[r, h * hd + (p, p + hd/2)] rotated (inverse: by the transpose) with the table
// cs[r * cs_ld + (p, hd/2 + p)] (rope.cu; dtype of x and cs alike)
int rope_apply_table(int dtype, int64_t rows, int heads, int hd, void* x, int64_t ldx,
                     const void* cs, int64_t cs_ld, int inverse, cudaStream_t st);

}  // namespace pe
