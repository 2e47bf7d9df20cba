/*
 * pe_b200.h -- C ABI of the B200 drafter-training-step library (libpe_b200.so).
 *
 * Plain pointers, int64 sizes/strides, a dtype code and a cudaStream_t (passed as
 * void*).  No entry point allocates device memory: callers pass every output and
 * workspace buffer.  Every entry point returns 0 on success or a nonzero PE_ERR_*
 * code; pe_last_error() then returns a message (thread-local).
 *
 * Kernels that wait on barriers (the tensor-core paths) bound every wait; a wait
 * that times out writes a nonzero code into the caller's `status` word (device
 * int32, may be NULL) and the kernel unwinds instead of hanging.
 *
 * Reference citations are to the Python reference project (puneethgv/parallel_eagle),
 * paths relative to its root; each entry point names the reference operation it
 * replaces.
 */
#ifndef PE_B200_H
#define PE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* dtype codes */
#define PE_F32 0
#define PE_BF16 1
#define PE_F16 2 /* source features only (pe_feature_norm_*): cached shards are fp16 */

/* error codes */
#define PE_OK 0
#define PE_ERR_ARG 1     /* invalid argument (shape, stride, alignment, dtype) */
#define PE_ERR_CUDA 2    /* a CUDA runtime/driver call failed */
#define PE_ERR_UNSUPPORTED 3
#define PE_ERR_WORKSPACE 4

/* algorithm selection for pe_gemm / pe_attn_* / pe_lmhead_ce */
#define PE_ALGO_AUTO 0
#define PE_ALGO_SIMT 1     /* fp32-FMA CUDA-core kernels (fp32 mode and odd shapes) */
#define PE_ALGO_TCGEN05 2  /* sm_100a tensor-core kernels (bf16) */

/* attention slot layouts (how the kernel re-derives the attend rule) */
#define PE_LAYOUT_PARTITION 0 /* real 0..a1-1, then anchors a0..a1-1 x depths 1..K-1 */
#define PE_LAYOUT_INDEXED 1   /* explicit int32 anchor[]/depth[] per slot */
#define PE_LAYOUT_BIAS 2      /* caller-supplied dense additive bias */

const char* pe_last_error(void);
int pe_version(void);
/* number of kernels this library launched since load (for launch accounting) */
int64_t pe_launch_count(void);

/* ---------------------------------------------------------------------------
 * RMSNorm  y = (x * rsqrt(mean(x^2) + eps)) * w, computed in fp32.
 * Replaces reference src/pe/nn.py:22-26 (RMSNorm.forward) and its autograd
 * backward.  rows x H, row strides ldx/ldy in elements.
 * ------------------------------------------------------------------------- */
int pe_rmsnorm_fwd(int dtype, int64_t rows, int64_t H, const void* x, int64_t ldx,
                   const void* w, void* y, int64_t ldy, float* rstd, float eps,
                   void* stream);
/* dx = (residual ? residual : 0) + d/dx ; dw_partial[nblk, H] (fp32) receives the
 * per-block partial of sum_rows dy * x * rstd (NULL to skip the weight gradient).
 * nblk is returned by pe_rmsnorm_bwd_blocks(rows). dx may alias residual. */
int pe_rmsnorm_bwd(int dtype, int64_t rows, int64_t H, const void* dy, int64_t lddy,
                   const void* x, int64_t ldx, const void* w, const float* rstd,
                   void* dx, int64_t lddx, const void* residual, int64_t ldres,
                   float* dw_partial, void* stream);
int64_t pe_rmsnorm_bwd_blocks(int64_t rows);
/* No counterpart in the reference.  For callers that cannot allocate device memory
 * (a host that owns the whole device budget, or a hot path where cudaMalloc's device
 * synchronisation is not allowed): the same dx as pe_rmsnorm_bwd plus
 * dw = (accumulate ? dw : 0) + sum_rows dy * x * rstd, with the per-block partials
 * kept in a 2 MiB array inside the library (H <= 8192; larger H is rejected with
 * PE_ERR_ARG).  The first call on a device looks the array up -- make it before any
 * stream capture.  Calls share the array: calls that overlap on the GPU race. */
int pe_rmsnorm_bwd_noalloc(int dtype, int64_t rows, int64_t H, const void* dy, int64_t lddy,
                           const void* x, int64_t ldx, const void* w, const float* rstd,
                           void* dx, int64_t lddx, const void* residual, int64_t ldres,
                           void* dw, int accumulate, void* stream);
/* Feature ingestion fused with the feature RMSNorm (reference src/pe/drafter.py:129-130:
 * features.to(dtype), viewed as [n, nfl, H], RMSNorm with one shared weight).  Output row
 * o = t * nfl + b (t < tokens, b < nfl) normalises block b of source row src_tok[t] (row
 * t when src_tok is NULL) of x (x_dtype: PE_F16, PE_BF16 or PE_F32, row stride ldx),
 * each element first rounded to dtype as the reference's cast rounds it; rstd[o] is
 * written.  H a multiple of 256 up to 8192, 16-byte aligned rows.  The step feeds every
 * stacked segment the real prefix rows this way, with no cast or gathered copy of the
 * shard.  pe_feature_norm_dw adds the weight gradient only (features take no gradient):
 * dw_partial[nblk, H] (nblk = pe_rmsnorm_bwd_blocks(tokens * nfl), reduce with
 * pe_colsum_f32) of sum_o dy[o] * x[o] * rstd[o], x read through the same map. */
int pe_feature_norm_fwd(int x_dtype, int dtype, int64_t tokens, int nfl, int64_t H,
                        const void* x, int64_t ldx, const int64_t* src_tok, const void* w,
                        void* y, int64_t ldy, float* rstd, float eps, void* stream);
int pe_feature_norm_dw(int x_dtype, int dtype, int64_t tokens, int nfl, int64_t H,
                       const void* dy, int64_t lddy, const void* x, int64_t ldx,
                       const int64_t* src_tok, const float* rstd, float* dw_partial,
                       void* stream);
/* dw (dtype) = (accumulate ? dw : 0) + sum over nblk partial rows */
int pe_colsum_f32(int dtype, int64_t nblk, int64_t H, const float* partial, void* dw,
                  int accumulate, void* stream);

/* ---------------------------------------------------------------------------
 * Rotary embedding, half-split (rotate_half), in place on `heads` consecutive
 * head_dim-wide column blocks of each row.  cos/sin from pos (int64) in fp32 and
 * rounded to dtype before use.  inverse=1 applies the transpose (backward).
 * Replaces reference src/pe/nn.py:29-49 (build_rope_cache + apply_rope).
 * ------------------------------------------------------------------------- */
int pe_rope(int dtype, int64_t rows, int heads, int head_dim, void* x, int64_t ldx,
            const int64_t* pos, float theta, int inverse, void* stream);
/* The cos / sin table the fused rotations read: row r (stride ld >= head_dim) holds
 * cos(pos[r] f_p) for p < head_dim/2, then sin(pos[r] f_p), rounded to dtype, with
 * the same angles and rounding as pe_rope (reference src/pe/nn.py:29-40,
 * build_rope_cache).  Positions are fixed per slot layout, so a caller builds the
 * table once per layout and reuses it. */
int pe_rope_table(int dtype, int64_t rows, int head_dim, const int64_t* pos, float theta,
                  void* cs, int64_t ld, void* stream);

/* ---------------------------------------------------------------------------
 * GEMM  C[m,n] = alpha * sum_k A(m,k) B(n,k) + beta * Cin[m,n]
 *   A(m,k) = A[m*a_sm + k*a_sk], B(n,k) = B[n*b_sn + k*b_sk], C row-major (ldc).
 * Covers nn.Linear forward (A=x, B=W), its input gradient and weight gradient
 * (reference src/pe/nn.py:66-69,75-80,89,95-100, src/pe/drafter.py:131-137).
 * Cin may alias C (in-place accumulation, e.g. into .grad).  c_dtype is the
 * dtype of C and Cin.
 * Tuning bits of `algo` above the algorithm code (0 = automatic for each):
 *   bits 8-17  tile width: 128/160/192/224/256 single-CTA, 128/192/256/384/512 pair
 *   bits 20-21 1 = single-CTA 128-row tiles, 2 = CTA-pair 256-row tiles (cta_group::2)
 *   bits 24-29 tile-group size of the L2-aware tile order; bit 30 groups N-tiles
 * ------------------------------------------------------------------------- */
int pe_gemm(int dtype, int64_t M, int64_t N, int64_t K, const void* A, int64_t a_sm,
            int64_t a_sk, const void* B, int64_t b_sn, int64_t b_sk, void* C, int64_t ldc,
            int c_dtype, const void* Cin, int64_t ldcin, float alpha, float beta, int algo,
            int32_t* status, void* stream);

/* y = x w^T (bf16; x [M, K], w [N, K], both row-major with unit column stride) with
 * the rotary embedding applied in the GEMM epilogue to the head_dim-wide column
 * blocks of [0, rot_cols) using the pe_rope_table table rope_cs (row m of the table
 * for row m of y): the fused q|k|v projection + RoPE of reference
 * src/pe/nn.py:75-80 (q/k/v_proj then apply_rope).  Bit-identical to pe_gemm
 * followed by pe_rope.  Tensor-core path only: dtype bf16, head_dim 128, N and
 * rot_cols multiples of 128, 16-byte aligned rows. */
int pe_linear_rope(int dtype, int64_t M, int64_t N, int64_t K, const void* x, int64_t ldx,
                   const void* w, int64_t ldw, void* y, int64_t ldy, const void* rope_cs,
                   int64_t cs_ld, int64_t rot_cols, int head_dim, int32_t* status,
                   void* stream);

/* gu = x w_gu^T ([M, 2I]: gate columns [0, I), up columns [I, 2I); w_gu rows [0, I)
 * gate_proj, [I, 2I) up_proj, all row-major with unit column stride) and
 * act = silu(gate) * up ([M, I]), each rounded to dtype as pe_gemm then
 * pe_swiglu_fwd would round them (bit-identical): the SwiGLU MLP's gate / up
 * projections and activation (reference src/pe/nn.py:99-100).  On the bf16
 * tensor-core path with CTA-pair tiles (M >= 512, I a multiple of half the tile
 * width) the activation is computed in the GEMM epilogue -- each tile loads
 * matching gate and up weight rows -- so gu is not re-read; otherwise the GEMM and
 * the element-wise kernel run back to back.  algo bits 8-17 may force the pair
 * tile width (256 or 512). */
int pe_linear_swiglu(int dtype, int64_t M, int64_t I, int64_t K, const void* x, int64_t ldx,
                     const void* w_gu, int64_t ldw, void* gu, int64_t ldgu, void* act,
                     int64_t lda, int algo, int32_t* status, void* stream);

/* The SwiGLU MLP's backward through the activation: d act = dy w (dy [M, K] the
 * down projection's output gradient, w = down_proj.weight [K, I], row stride ldw)
 * and dgu = swiglu_backward(d act, gu) ([M, 2I]: d gate | d up, with gu the
 * forward's gate | up rows), each rounded as pe_gemm then pe_swiglu_bwd would
 * round them (bit-identical).  Replaces the backward of reference
 * src/pe/nn.py:99-100 (down_proj input gradient, then silu(gate) * up).  On the
 * bf16 tensor-core path with CTA-pair tiles (M >= 512, I a multiple of 32, 16-byte
 * aligned rows) the SwiGLU backward runs in the GEMM epilogue and d act is never
 * stored; otherwise the GEMM writes d act into dgu's up half and pe_swiglu_bwd
 * rewrites dgu in place.  dgu must not alias gu.  algo bits 8-17 may force the pair
 * tile width (256 or 512). */
int pe_linear_swiglu_bwd(int dtype, int64_t M, int64_t I, int64_t K, const void* dy,
                         int64_t lddy, const void* w, int64_t ldw, const void* gu, int64_t ldgu,
                         void* dgu, int64_t lddgu, int algo, int32_t* status, void* stream);

/* ---------------------------------------------------------------------------
 * Cross-depth masked attention (GQA, scale = 1/sqrt(head_dim)), flash-style:
 * no score matrix is materialised.  q/k/v/o rows are slots, heads are
 * head_dim-wide column blocks; per-batch strides *_sb, per-slot strides *_ss.
 * lse[b, h, s] (fp32) is written by fwd and read by bwd.
 * Layout PARTITION uses (a0, a1, kdepth); INDEXED uses anchor/depth[S];
 * BIAS uses bias (dtype) with batch stride bias_sb (0 = broadcast) and row
 * stride bias_sq.
 * Replaces reference src/pe/nn.py:71-89 (Attention core + repeat_kv) with the mask
 * of src/pe/masks.py:43-61 / partition.py:41-55,97.
 * ------------------------------------------------------------------------- */
int pe_attn_fwd(int dtype, int64_t B, int64_t S, int Hq, int Hkv, int head_dim,
                const void* q, int64_t q_sb, int64_t q_ss, const void* k, int64_t k_sb,
                int64_t k_ss, const void* v, int64_t v_sb, int64_t v_ss, void* o,
                int64_t o_sb, int64_t o_ss, float* lse, int layout, int64_t a0, int64_t a1,
                int kdepth, const int32_t* anchor, const int32_t* depth, const void* bias,
                int64_t bias_sb, int64_t bias_sq, int algo, int32_t* status, void* stream);
/* dq/dk/dv are overwritten.  `workspace` holds per-row softmax deltas and, on
 * the tensor-core path, fp32 dQ / dK / dV accumulators and a work counter; its
 * size comes from pe_attn_bwd_workspace (same shape arguments).  On the
 * tensor-core path, algo bits 8-15 pick the kernel variant: 0 (default) a dQ
 * kernel plus a persistent dK/dV kernel, 1 one fused kernel with dQ atomics,
 * 2 a dQ kernel plus one dK/dV CTA per key tile.  The forward's bits 8-15: 0
 * (default) two query tiles per CTA, 1 one. */
size_t pe_attn_bwd_workspace(int dtype, int64_t B, int64_t S, int Hq, int Hkv, int head_dim);
int pe_attn_bwd(int dtype, int64_t B, int64_t S, int Hq, int Hkv, int head_dim,
                const void* q, int64_t q_sb, int64_t q_ss, const void* k, int64_t k_sb,
                int64_t k_ss, const void* v, int64_t v_sb, int64_t v_ss, const void* o,
                int64_t o_sb, int64_t o_ss, const void* dout, int64_t do_sb, int64_t do_ss,
                const float* lse, void* dq, int64_t dq_sb, int64_t dq_ss, void* dk,
                int64_t dk_sb, int64_t dk_ss, void* dv, int64_t dv_sb, int64_t dv_ss,
                void* workspace, size_t workspace_bytes, int layout, int64_t a0, int64_t a1,
                int kdepth, const int32_t* anchor, const int32_t* depth, const void* bias,
                int64_t bias_sb, int64_t bias_sq, int algo, int32_t* status, void* stream);

/* ---------------------------------------------------------------------------
 * Masked attention over all segments of one sequence in one call (partition
 * layout).  Segment s spans anchors [a0, a1) = (bounds[2s], bounds[2s + 1]) and
 * has S_s = a1 + (a1 - a0)(kdepth - 1) slots, stored in rows
 * [row0_s, row0_s + S_s) of every row operand with row0_0 = 0 and
 * row0_{s+1} = row0_s + S_s (the segments stacked one after another).  lse
 * (and the backward's deltas) hold one [Hq, S_s] fp32 block per segment,
 * starting at element Hq * row0_s.  On the tensor-core path one launch per
 * kernel covers every segment (the largest segment's units first, heaviest
 * first within a segment, so a segment's tail overlaps the next segment's
 * start); otherwise the segments run one after another.  Kernel-variant bits
 * are not accepted here.  Results equal per-segment pe_attn_fwd / pe_attn_bwd
 * calls.  Replaces the per-segment attention of reference
 * src/pe/partition.py:86-117 (one ParallelDrafter.forward / backward per
 * segment, each reaching src/pe/nn.py:71-89).
 * ------------------------------------------------------------------------- */
int pe_attn_fwd_segments(int dtype, int nseg, const int64_t* bounds, int kdepth, int Hq,
                         int Hkv, int head_dim, const void* q, int64_t q_ss, const void* k,
                         int64_t k_ss, const void* v, int64_t v_ss, void* o, int64_t o_ss,
                         float* lse, int algo, int32_t* status, void* stream);
size_t pe_attn_bwd_segments_workspace(int dtype, int nseg, const int64_t* bounds, int kdepth,
                                      int Hq, int Hkv, int head_dim);
/* rope_cs (may be NULL): a pe_rope_table table with one row per stacked slot row
 * (row stride cs_ld elements, dtype as the operands).  With it q and k are the
 * rotated projections and dq / dk are returned rotated back by the transpose of the
 * rotary embedding -- the gradients with respect to the unrotated projections, as
 * pe_rope(inverse = 1) on the plain result would give, bit for bit.  On the
 * tensor-core path the rotation is fused into the dQ store and the dK cast. */
int pe_attn_bwd_segments(int dtype, int nseg, const int64_t* bounds, int kdepth, int Hq,
                         int Hkv, int head_dim, const void* q, int64_t q_ss, const void* k,
                         int64_t k_ss, const void* v, int64_t v_ss, const void* o,
                         int64_t o_ss, const void* dout, int64_t do_ss, const float* lse,
                         void* dq, int64_t dq_ss, void* dk, int64_t dk_ss, void* dv,
                         int64_t dv_ss, void* workspace, size_t workspace_bytes,
                         const void* rope_cs, int64_t cs_ld, int algo, int32_t* status,
                         void* stream);

/* ---------------------------------------------------------------------------
 * Frozen shared LM head fused with the loss and its input gradient, chunked
 * over the vocabulary: logits for the whole vocabulary are never stored.
 *   z = h W^T (rounded to dtype), loss_r = lse(z_r) - z_r[label_r]
 *   (or, with teacher rows t_r: loss_r = -sum_v softmax(t_r W^T)_v log_softmax(z_r)_v)
 *   loss_sum[0] += sum_r loss_r;  dh = grad_scale * d(sum_r loss_r)/dh
 * Rows with label < 0 are ignored.  No gradient reaches W (frozen).
 * For the bf16 paths, algo bits 8-15 set the vocabulary chunk (units of 1024 rows
 * of W, at most 32) and bits 16-23 the
 * loss-row group (units of 256 rows, at most 40); zero keeps the defaults (32768
 * and 10240).  Bits 24-25 / 26-27 pick the logits / dH GEMM
 * tile width (1: 256, 2: 512, 0: automatic).  On both bf16 paths every vocabulary
 * chunk after a row group's first is one pass (the logits GEMMs write e^(z - running
 * max) directly; a logit more than 64 above its row's running maximum makes the call
 * recompute itself two-pass on the device); bit 28 runs every chunk two-pass.
 * Replaces reference src/pe/partition.py:113-115 (lm_head -> float ->
 * cross_entropy(sum) -> backward) and drafter.py:123-124.
 * ------------------------------------------------------------------------- */
size_t pe_lmhead_ce_workspace(int dtype, int64_t R, int64_t H, int64_t V, int soft);
int pe_lmhead_ce(int dtype, int64_t R, int64_t H, int64_t V, const void* h, int64_t ldh,
                 const void* W, const int64_t* labels, const void* teacher, int64_t ldt,
                 float grad_scale, void* dh, int64_t lddh, float* loss_sum, void* workspace,
                 size_t workspace_bytes, int algo, int32_t* status, void* stream);

/* ---------------------------------------------------------------------------
 * Small fused pieces of the drafter input / MLP (reference src/pe/drafter.py:126-137,
 * src/pe/nn.py:99-100).
 * ------------------------------------------------------------------------- */
/* out[r, 0:H] = embed[ids[r], :] (embed dtype = dtype) */
int pe_embed_rows(int dtype, int64_t rows, int64_t H, const int64_t* ids, const void* embed,
                  void* out, int64_t ldo, void* stream);
/* out[r, :] = vec for rows r in [0, rows) */
int pe_fill_rows(int dtype, int64_t rows, int64_t H, const void* vec, void* out, int64_t ldo,
                 void* stream);
/* a = silu(g) * u with g = gu[:, 0:I], u = gu[:, I:2I] (each rounded to dtype) */
int pe_swiglu_fwd(int dtype, int64_t rows, int64_t I, const void* gu, int64_t ldgu, void* a,
                  int64_t lda, void* stream);
/* dgu[:, 0:I] = da*u*silu'(g), dgu[:, I:2I] = da*silu(g) */
int pe_swiglu_bwd(int dtype, int64_t rows, int64_t I, const void* da, int64_t ldda,
                  const void* gu, int64_t ldgu, void* dgu, int64_t lddgu, void* stream);
/* out[c] (fp32) = sum_r x[r, c] (overwrite) */
int pe_rowsum_cols(int dtype, int64_t rows, int64_t H, const void* x, int64_t ldx, float* out,
                   void* stream);
/* out[c] (fp32) = sum over rows r of the nranges (1..16) host-side [begin, end) pairs in
 * `ranges` of x[r, c] (overwrite), in a fixed order: the expand backward of the shared
 * prediction-slot input over every segment's prediction rows in one launch (reference
 * src/pe/drafter.py:137).  Rows of overlapping ranges count once per range. */
int pe_rowsum_cols_ranges(int dtype, int nranges, const int64_t* ranges, int64_t H,
                          const void* x, int64_t ldx, float* out, void* stream);
/* dst[idx[r], :] = src[r, :] (scatter, dst rows not listed are left untouched) and the
 * inverse gather dst[r, :] = src[idx[r], :] */
int pe_scatter_rows(int dtype, int64_t rows, int64_t H, const int64_t* idx, const void* src,
                    int64_t lds, void* dst, int64_t ldd, void* stream);
int pe_gather_rows(int dtype, int64_t rows, int64_t H, const int64_t* idx, const void* src,
                   int64_t lds, void* dst, int64_t ldd, void* stream);
/* y (dtype) = x (fp32) elementwise cast, n elements */
int pe_cast_f32(int dtype, int64_t n, const float* x, void* y, void* stream);

/* ---------------------------------------------------------------------------
 * Draft-time selection: per row of logits (dtype, row stride ld), the log-
 * probabilities lp = (z - max z) - log(sum exp(z - max z)) in fp32 (raw = 1:
 * the logits themselves) and the k best columns in order (value descending,
 * then column ascending): idx[r, 0..k) (int64), val[r, 0..k) (fp32).  Replaces
 * log_softmax(logits.float()).topk of reference src/pe/decode/tree.py:33-41 and
 * logits.argmax of src/pe/decode/chain.py:22-23 / src/pe/drafter.py:268.
 * ------------------------------------------------------------------------- */
int pe_topk_logprobs(int dtype, int64_t rows, int64_t V, const void* logits, int64_t ld, int k,
                     int raw, int64_t* idx, float* val, void* stream);
/* q[r, v] (fp32, row stride ldq) = softmax(z[r, :] / temperature)[v] in fp32 for
 * logits z (dtype, row stride ld): the per-depth sampling distributions of
 * reference src/pe/decode/chain.py:50 (torch.softmax(logits.float() / temperature)).
 * temperature must be positive and finite. */
int pe_softmax_rows(int dtype, int64_t rows, int64_t V, const void* logits, int64_t ld,
                    float temperature, float* q, int64_t ldq, void* stream);

/* ---------------------------------------------------------------------------
 * Optimizer (reference src/pe/train.py:26-34,158-159: clip_grad_norm_(1.0) then
 * AdamW.step()).  sumsq_out (fp32 [1]) += sum g^2; the step reads it to apply the
 * clipping coefficient min(1, max_norm / (sqrt(sumsq) + 1e-6)).
 * m, v are fp32 moment buffers.
 * ------------------------------------------------------------------------- */
int pe_sumsq(int dtype, int64_t n, const void* g, float* sumsq_out, void* stream);
/* The same sum of squares, deterministic: partials[b] (fp32, b < nblk <= 65535) =
 * block b's share over a fixed grid of nblk blocks, no atomics; pe_sum_f32 then adds
 * n floats in a fixed order into out[0] (accumulate = 1: out[0] += the sum).  Used for
 * the global-norm clip of data-parallel updates, so every rank holding the same
 * gradient computes the same coefficient (pe_sumsq's atomic order varies from run to
 * run and rank to rank). */
int pe_sumsq_partials(int dtype, int64_t n, const void* g, float* partials, int64_t nblk,
                      void* stream);
int pe_sum_f32(int64_t n, const float* x, float* out, int accumulate, void* stream);
int pe_adamw_step(int dtype, int64_t n, void* p, const void* g, float* m, float* v,
                  const float* sumsq, float max_norm, float lr, float beta1, float beta2,
                  float eps, float weight_decay, int64_t step, void* stream);

/* ---------------------------------------------------------------------------
 * Self-test of the bounded-wait unwind path (no counterpart in the reference).
 * One warp allocates tensor memory, waits on an mbarrier that nothing arrives at,
 * gives up after limit_ns (1 us .. 10 s), writes code 901 into *status (first
 * writer wins, as in every tensor-core kernel), frees its tensor memory and
 * returns; *waited_out = 1 if the wait ran out.  The tensor-core kernels use the
 * same wait with a 4 s limit.
 * ------------------------------------------------------------------------- */
int pe_wait_probe(uint64_t limit_ns, int32_t* status, int32_t* waited_out, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* PE_B200_H */
