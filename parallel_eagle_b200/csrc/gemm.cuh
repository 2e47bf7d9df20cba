// Internal GEMM entry points shared by the dispatcher, the LM-head loss and
// the attention code.
#pragma once
#include "common.cuh"

namespace pe {

int gemm_simt(int dtype, int64_t M, int64_t N, int64_t K, const void* A, int64_t a_sm,
              int64_t a_sk, const void* B, int64_t b_sn, int64_t b_sk, void* C, int64_t ldc,
              int c_dtype, const void* Cin, int64_t ldcin, float alpha, float beta,
              cudaStream_t stream);

// True when the tcgen05/TMA kernel can take these operands (bf16, unit stride on
// one side of each operand, 16-byte aligned strides and bases).
bool gemm_tc_eligible(int dtype, int64_t M, int64_t N, int64_t K, const void* A, int64_t a_sm,
                      int64_t a_sk, const void* B, int64_t b_sn, int64_t b_sk, int c_dtype);

int gemm_tc(int64_t M, int64_t N, int64_t K, const void* A, int64_t a_sm, int64_t a_sk,
            const void* B, int64_t b_sn, int64_t b_sk, void* C, int64_t ldc, int c_dtype,
            const void* Cin, int64_t ldcin, float alpha, float beta, int* status,
            cudaStream_t stream, int force_bn = 0, int mode = 0, int raster = 0,
            int store_hint = 0);

// Logits GEMM for the fused LM-head loss: C (bf16, [M, N]) = A[M, K] B[N, K]^T with
// both operands K-major, and per (row, 128-column chunk) the pair (max, sum exp(c - max))
// of the stored (rounded) values in stats[row * stats_ld + tile].  A non-null run_if
// whose word is 0 makes the launch do nothing (likewise below).
int gemm_tc_logits_stats(int64_t M, int64_t N, int64_t K, const void* A, int64_t lda,
                         const void* B, int64_t ldb, void* C, int64_t ldc, float2* stats,
                         int stats_ld, int* status, cudaStream_t stream, int force_bn = 0,
                         const int* run_if = nullptr);

// The same logits written as P = e^(z - rowref[row]) (bf16; 0 for rows whose label is
// negative) with per-128-column (max z, sum P) pairs, the label logit z[labels[r] -
// label_v0] of rows whose label falls in these columns (labels may be null: no row
// ignored, no label logit), and *overflow = 1 when some z
// exceeds its row's reference by more than 64 (P would leave the fp32 range).
int gemm_tc_logits_pexp(int64_t M, int64_t N, int64_t K, const void* A, int64_t lda,
                        const void* B, int64_t ldb, void* P, int64_t ldp, float2* stats,
                        int stats_ld, const float* rowref, const int64_t* labels,
                        int64_t label_v0, float* zlab, int* overflow, int* status,
                        cudaStream_t stream, int force_bn = 0);

// C (fp32) = A[M, K] B + rowscale[row] * Cin, A K-major, B (n, k) at B[n + k * b_sk]
// (MN-major): the online-softmax rescaled accumulation of the LM-head input gradient.
int gemm_tc_rowscale_acc(int64_t M, int64_t N, int64_t K, const void* A, int64_t lda,
                         const void* B, int64_t b_sk, float* C, int64_t ldc, const float* Cin,
                         const float* rowscale, int* status, cudaStream_t stream,
                         int force_bn = 0, const int* run_if = nullptr);

// pe_gemm without the C wrapper (used inside the library)
int gemm(int dtype, int64_t M, int64_t N, int64_t K, const void* A, int64_t a_sm, int64_t a_sk,
         const void* B, int64_t b_sn, int64_t b_sk, void* C, int64_t ldc, int c_dtype,
         const void* Cin, int64_t ldcin, float alpha, float beta, int algo, int* status,
         cudaStream_t stream);

}  // namespace pe
