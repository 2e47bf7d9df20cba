"""Per-kernel parity on the GPU: each libpe_b200 entry point against a plain
PyTorch fp32 reference of the same op (bf16 inputs are rounded first, so the
reference sees exactly what the kernel sees)."""

from __future__ import annotations

import math

import pytest
import torch

from gpu_harness import oracle, recipe

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover - collected on CPU boxes too
    pytest.skip("needs a CUDA device", allow_module_level=True)

from parallel_eagle_b200 import _lib as L  # noqa: E402
from parallel_eagle_b200 import ops  # noqa: E402

DEV = torch.device("cuda")
rel = recipe.rel_fro


def _rand(*shape, dtype=torch.bfloat16, scale=1.0, seed=0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(dtype).to(DEV)


def _pad8(x):
    return (x + 7) // 8 * 8


# ------------------------------------------------------------------ GEMM ----


def _operand(rows, cols, mn_major, dtype, seed):
    """Logical [rows, cols] operand (rows = M or N, cols = K); returns the tensor,
    (stride_row, stride_k) and the dense logical fp32 view."""
    g = torch.Generator().manual_seed(seed)
    dense = torch.randn(rows, cols, generator=g).to(dtype)
    if not mn_major:
        ld = _pad8(cols)
        store = torch.zeros(rows, ld, dtype=dtype)
        store[:, :cols] = dense
        return store.to(DEV), (ld, 1), dense.float()
    ld = _pad8(rows)
    store = torch.zeros(cols, ld, dtype=dtype)
    store[:, :rows] = dense.t()
    return store.to(DEV), (1, ld), dense.float()


@pytest.mark.parametrize("shape", [(128, 256, 64), (300, 200, 136), (1, 512, 256),
                                   (257, 129, 1000), (512, 640, 384)])
@pytest.mark.parametrize("a_mn", [False, True])
@pytest.mark.parametrize("b_mn", [False, True])
@pytest.mark.parametrize("out_f32", [False, True])
@pytest.mark.parametrize("mode", [1, 2])  # 1: single-CTA tiles, 2: CTA-pair (cta_group::2) tiles
def test_gemm_tcgen05_matches_fp32(shape, a_mn, b_mn, out_f32, mode):
    M, N, K = shape
    algo = L.ALGO_TCGEN05 | (mode << 20)
    A, (a_sm, a_sk), Ad = _operand(M, K, a_mn, torch.bfloat16, 1)
    B, (b_sn, b_sk), Bd = _operand(N, K, b_mn, torch.bfloat16, 2)
    cdt = torch.float32 if out_f32 else torch.bfloat16
    ldc = _pad8(N)
    C = torch.full((M, ldc), 7.0, dtype=cdt, device=DEV)
    ref = Ad @ Bd.t()
    ops.gemm(M, N, K, A, a_sm, a_sk, B, b_sn, b_sk, C, ldc, algo=algo)
    torch.cuda.synchronize()
    ops.check_status(DEV)
    got = C[:, :N].float().cpu()
    assert rel(got, ref) < (1e-5 if out_f32 else 5e-3)
    assert torch.all(C[:, N:].float() == 7.0)  # untouched padding
    # accumulate: C = 0.5 * A B^T + 1.0 * C
    prev = C[:, :N].float().cpu().clone()
    ops.gemm(M, N, K, A, a_sm, a_sk, B, b_sn, b_sk, C, ldc, Cin=C, ldcin=ldc, alpha=0.5,
             beta=1.0, algo=algo)
    torch.cuda.synchronize()
    assert rel(C[:, :N].float().cpu(), prev + 0.5 * ref) < (1e-5 if out_f32 else 5e-3)


@pytest.mark.parametrize("bn", [128, 160, 192, 224, 256])
@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (True, False), (False, True), (True, True)])
def test_gemm_tcgen05_every_tile_width(bn, a_mn, b_mn):
    if b_mn and bn % 64:
        pytest.skip("MN-major B needs a tile width that is a multiple of 64")
    M, N, K = 300, 3584 // 4 + 40, 520
    A, (a_sm, a_sk), Ad = _operand(M, K, a_mn, torch.bfloat16, 5)
    B, (b_sn, b_sk), Bd = _operand(N, K, b_mn, torch.bfloat16, 6)
    C = torch.zeros(M, N, dtype=torch.float32, device=DEV)
    ops.gemm(M, N, K, A, a_sm, a_sk, B, b_sn, b_sk, C, N, algo=L.ALGO_TCGEN05 | (bn << 8))
    torch.cuda.synchronize()
    ops.check_status(DEV)
    assert rel(C.cpu(), Ad @ Bd.t()) < 1e-5


@pytest.mark.parametrize("bn", [128, 192, 256, 384, 512])
@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (True, False), (False, True), (True, True)])
@pytest.mark.parametrize("M", [300, 1100])
def test_gemm_tcgen05_pair_tile_widths(bn, a_mn, b_mn, M):
    # CTA-pair tiles (256 x bn; above 256 two MMAs per K step into one 512-column
    # accumulator): ragged M leaves the second CTA's rows partly or wholly outside the
    # matrix; ragged N leaves part of the last tile's B sub-tiles empty
    b_rows = (bn // 2 if bn > 256 else bn) // 2  # B rows of one MMA held by each CTA
    if b_mn and b_rows % 64:
        pytest.skip("MN-major B needs 64-column B sub-tiles")
    N, K = 3584 // 4 + 40, 520
    A, (a_sm, a_sk), Ad = _operand(M, K, a_mn, torch.bfloat16, 7)
    B, (b_sn, b_sk), Bd = _operand(N, K, b_mn, torch.bfloat16, 8)
    C = torch.zeros(M, N, dtype=torch.float32, device=DEV)
    ops.gemm(M, N, K, A, a_sm, a_sk, B, b_sn, b_sk, C, N,
             algo=L.ALGO_TCGEN05 | (bn << 8) | (2 << 20))
    torch.cuda.synchronize()
    ops.check_status(DEV)
    assert rel(C.cpu(), Ad @ Bd.t()) < 1e-5


@pytest.mark.parametrize("mode", [1, 2])
@pytest.mark.parametrize("raster", [1, 3, 64 - 1, -1, -2, -5])
def test_gemm_tcgen05_tile_orders(mode, raster):
    # every tile order (groups of M-tiles or of N-tiles, ragged last group) covers
    # each output tile exactly once
    M, N, K = 1300, 2000, 200
    A, (a_sm, a_sk), Ad = _operand(M, K, False, torch.bfloat16, 9)
    B, (b_sn, b_sk), Bd = _operand(N, K, True, torch.bfloat16, 10)
    C = torch.full((M, N), float("nan"), dtype=torch.float32, device=DEV)
    bits = ((abs(raster) & 0x3F) << 24) | ((1 << 30) if raster < 0 else 0)
    ops.gemm(M, N, K, A, a_sm, a_sk, B, b_sn, b_sk, C, N,
             algo=L.ALGO_TCGEN05 | (mode << 20) | bits)
    torch.cuda.synchronize()
    ops.check_status(DEV)
    assert not torch.isnan(C).any()
    assert rel(C.cpu(), Ad @ Bd.t()) < 1e-5


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, True)])
def test_gemm_simt_matches_fp32(dtype, a_mn, b_mn):
    M, N, K = 77, 45, 133
    A, (a_sm, a_sk), Ad = _operand(M, K, a_mn, dtype, 3)
    B, (b_sn, b_sk), Bd = _operand(N, K, b_mn, dtype, 4)
    C = torch.empty(M, N, dtype=dtype, device=DEV)
    ops.gemm(M, N, K, A, a_sm, a_sk, B, b_sn, b_sk, C, N, algo=L.ALGO_SIMT)
    torch.cuda.synchronize()
    assert rel(C.float().cpu(), Ad @ Bd.t()) < (1e-6 if dtype == torch.float32 else 5e-3)


def test_gemm_rejects_ineligible_tcgen05():
    A = torch.zeros(16, 10, dtype=torch.bfloat16, device=DEV)  # row stride 10 elements: not 16 B
    C = torch.zeros(16, 16, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(L.PeError):
        ops.gemm(16, 16, 10, A, 10, 1, A, 10, 1, C, 16, algo=L.ALGO_TCGEN05)


# --------------------------------------------------------------- RMSNorm ----


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("H,rows", [(64, 37), (3584, 37), (100, 37), (3584, 5003), (4096, 700),
                                    (512, 300), (1536, 1000), (5120, 257)])
@pytest.mark.parametrize("with_res", [True, False])
def test_rmsnorm_fwd_bwd(dtype, H, rows, with_res):
    # 5003 rows: more row tiles than persistent blocks, ragged last tile; H = 512 m <= 4096
    # takes the one-block-per-row bf16 kernel, 5120 the tiled one
    x = _rand(rows, H, dtype=dtype, seed=5) * 3
    w = (1 + 0.1 * _rand(H, dtype=torch.float32, seed=6)).to(dtype)
    dy = _rand(rows, H, dtype=dtype, seed=7)
    res = _rand(rows, H, dtype=dtype, seed=8) if with_res else torch.zeros(rows, H, dtype=dtype,
                                                                            device=DEV)
    y, rstd = ops.rmsnorm_fwd(x, w, 1e-5)
    xr = x.float().cpu().requires_grad_(True)
    wr = w.float().cpu().requires_grad_(True)
    yr = oracle.rms_norm(xr, wr, 1e-5)
    tol = 1e-6 if dtype == torch.float32 else 1e-2
    assert rel(y.float().cpu(), yr) < tol
    yr.backward(dy.float().cpu())
    dx, part = ops.rmsnorm_bwd(dy, x, w, rstd, residual=res if with_res else None)
    dw = ops.colsum_into(part, torch.zeros(H, dtype=torch.float32, device=DEV), accumulate=False)
    torch.cuda.synchronize()
    assert rel(dx.float().cpu() - res.float().cpu(), xr.grad) < (1e-5 if dtype == torch.float32 else 2e-2)
    assert rel(dw.cpu(), wr.grad) < 1e-5


# ------------------------------------------------------------------ RoPE ----


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("max_pos", [256, 12000])
def test_rope_matches_reference_rotation(dtype, max_pos):
    # fp32 tolerance grows with the position: the angle pos * inv_freq is an fp32
    # product (as in the reference), so one ulp of inv_freq between two libms moves
    # it by ~pos * 6e-8 rad.
    S, heads, hd = 50, 6, 64
    x = _rand(S, heads * hd + 16, dtype=dtype, seed=9)  # extra columns stay untouched
    pos = torch.randint(0, max_pos, (S,), generator=torch.Generator().manual_seed(1)).to(DEV)
    y = x.clone()
    ops.rope_(y, heads, hd, pos, 10000.0)
    cos, sin = oracle.rope_tables(pos.cpu(), hd, 10000.0)
    xh = x[:, : heads * hd].cpu().view(S, heads, hd).transpose(0, 1)
    ref = oracle.drafter_step._rotate(xh, cos, sin).transpose(0, 1).reshape(S, heads * hd)
    tol = (2e-5 if max_pos <= 256 else 3e-4) if dtype == torch.float32 else 1e-2
    assert rel(y[:, : heads * hd].float().cpu(), ref.float()) < tol
    assert torch.equal(y[:, heads * hd:], x[:, heads * hd:])
    ops.rope_(y, heads, hd, pos, 10000.0, inverse=True)
    assert rel(y.float().cpu(), x.float().cpu()) < (1e-5 if dtype == torch.float32 else 2e-2)


@pytest.mark.parametrize("M,N,K", [(300, 640, 256), (1024, 1536, 512)])
@pytest.mark.parametrize("out_f32", [False, True])
def test_gemm_evict_first_stores_match_plain(M, N, K, out_f32):
    """algo bit 22 (C stored with the L2 evict-first policy) changes only the cache
    policy: the results equal the plain GEMM's, accumulate included."""
    x = _rand(M, K, seed=72)
    w = _rand(N, K, seed=73, scale=0.05)
    dt = torch.float32 if out_f32 else torch.bfloat16
    base = _rand(M, N, dtype=dt, seed=74)
    ref = base.clone()
    ops.gemm(M, N, K, x, K, 1, w, K, 1, ref, N, Cin=ref, ldcin=N, alpha=0.5, beta=1.0,
             algo=L.ALGO_TCGEN05)
    got = base.clone()
    ops.gemm(M, N, K, x, K, 1, w, K, 1, got, N, Cin=got, ldcin=N, alpha=0.5, beta=1.0,
             algo=L.ALGO_TCGEN05 | (1 << 22))
    torch.cuda.synchronize()
    ops.check_status(DEV)
    assert torch.equal(got, ref)


@pytest.mark.parametrize("M,I,K,bn", [(300, 512, 256, 0), (600, 512, 320, 256), (600, 1024, 256, 512),
                                      (4096, 2048, 512, 0), (1500, 768, 192, 256)])
def test_linear_swiglu_equals_linear_then_swiglu(M, I, K, bn):
    """gate|up GEMM with silu(gate) * up in the epilogue (256- and 512-wide CTA-pair
    tiles; below 512 rows the plain GEMM + element-wise kernel) equals the plain GEMM
    followed by the SwiGLU kernel bit for bit, for both outputs."""
    x = _rand(M, K, seed=70)
    w = _rand(2 * I, K, seed=71, scale=0.05)
    gu_ref = ops.linear(x, w, algo=L.ALGO_TCGEN05)
    act_ref = ops.swiglu_fwd(gu_ref, I)
    gu, act = ops.linear_swiglu(x, w, I, algo=L.ALGO_AUTO | (bn << 8))
    torch.cuda.synchronize()
    ops.check_status(DEV)
    assert torch.equal(gu, gu_ref)
    assert torch.equal(act, act_ref)


@pytest.mark.parametrize("M,I,K,bn,dtype", [(300, 512, 256, 0, torch.bfloat16),
                                             (600, 512, 320, 256, torch.bfloat16),
                                             (600, 1024, 256, 512, torch.bfloat16),
                                             (4096, 2048, 512, 0, torch.bfloat16),
                                             (1500, 768, 192, 256, torch.bfloat16),
                                             (700, 520, 256, 0, torch.bfloat16),
                                             (600, 512, 256, 0, torch.float32)])
def test_linear_swiglu_bwd_equals_dgrad_then_swiglu_bwd(M, I, K, bn, dtype):
    """The down projection's input gradient with the SwiGLU backward in the GEMM
    epilogue (256- and 512-wide CTA-pair tiles, a ragged last row tile) equals the plain
    GEMM followed by the element-wise SwiGLU backward bit for bit; below 512 rows, with
    I not a multiple of 32 or in fp32 the entry point runs that pair itself (the GEMM
    writing into dgu's up half, the SwiGLU backward in place)."""
    dy = _rand(M, K, seed=72, dtype=dtype)
    w = _rand(K, I, seed=73, scale=0.05, dtype=dtype)
    gu = _rand(M, 2 * I, seed=74, dtype=dtype)
    ref = ops.swiglu_bwd(ops.linear_dgrad(dy, w), gu, I)
    got = ops.linear_swiglu_bwd(dy, w, gu, I, algo=L.ALGO_AUTO | (bn << 8))
    torch.cuda.synchronize()
    ops.check_status(DEV)
    assert torch.equal(got, ref)


@pytest.mark.parametrize("M,nh,nkv,K", [(200, 4, 2, 256), (700, 4, 2, 320), (1024, 28, 4, 512),
                                        (1300, 8, 2, 384)])
def test_linear_rope_equals_linear_then_rope(M, nh, nkv, K):
    """The q|k|v projection with RoPE in the GEMM epilogue (single-CTA and CTA-pair
    tiles, 256 and 512 wide) equals the plain GEMM followed by the rotation kernel,
    bit for bit; the v heads are left unrotated."""
    hd = 128
    N = (nh + 2 * nkv) * hd
    x = _rand(M, K, seed=60)
    w = _rand(N, K, seed=61, scale=0.05)
    pos = torch.randint(0, 9000, (M,), generator=torch.Generator().manual_seed(62)).to(DEV)
    ref = ops.linear(x, w, algo=L.ALGO_TCGEN05)
    ops.rope_(ref, nh + nkv, hd, pos, 10000.0)
    cs = ops.rope_table(pos, hd, 10000.0, torch.bfloat16)
    got = ops.linear_rope(x, w, cs, (nh + nkv) * hd, hd)
    torch.cuda.synchronize()
    ops.check_status(DEV)
    assert torch.equal(got, ref)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("case", [(300, 4, 5, 4, 2), (2048, 4, 5, 28, 4)])
def test_attention_bwd_fused_rope_equals_separate_rotation(case, dtype):
    """``attn_bwd_segments(rope_cs=...)`` (the transpose of RoPE fused into the dQ
    store and the dK cast, or a table pass on the CUDA-core path) equals the plain
    backward followed by the inverse rotation kernel: dQ bit for bit, dK and dV up
    to the order of the fp32 atomic GQA-group additions (not reproducible bit for bit
    from run to run)."""
    from parallel_eagle_b200.engine import segment_bounds

    n, nseg, k, nh, nkv = case
    if dtype == torch.float32 and n > 1000:
        pytest.skip("CUDA-core fp32 path: small cases only")
    hd = 128
    bounds = segment_bounds(n, nseg)
    R = sum(ops.segment_rows(bounds, k))
    cq, ckv = nh * hd, nkv * hd
    qkv = _rand(R, cq + 2 * ckv, dtype=dtype, seed=63)
    do = _rand(R, cq, dtype=dtype, seed=64)
    q, kt, vt = qkv[:, :cq], qkv[:, cq:cq + ckv], qkv[:, cq + ckv:]
    pos = torch.randint(0, 4096, (R,), generator=torch.Generator().manual_seed(65)).to(DEV)
    o, lse = ops.attn_fwd_segments(q, kt, vt, nh, nkv, hd, bounds, k)
    ref = torch.empty_like(qkv)
    ops.attn_bwd_segments(q, kt, vt, o, do, lse, nh, nkv, hd, bounds, k, dq=ref[:, :cq],
                          dk=ref[:, cq:cq + ckv], dv=ref[:, cq + ckv:])
    ops.rope_(ref, nh + nkv, hd, pos, 10000.0, inverse=True)
    cs = ops.rope_table(pos, hd, 10000.0, dtype)
    got = torch.full_like(qkv, float("nan"))
    ops.attn_bwd_segments(q, kt, vt, o, do, lse, nh, nkv, hd, bounds, k, dq=got[:, :cq],
                          dk=got[:, cq:cq + ckv], dv=got[:, cq + ckv:], rope_cs=cs)
    torch.cuda.synchronize()
    ops.check_status(DEV)
    assert torch.equal(got[:, :cq], ref[:, :cq])
    assert not torch.isnan(got).any()
    for sl in (slice(cq, cq + ckv), slice(cq + ckv, None)):
        assert rel(got[:, sl].float().cpu(), ref[:, sl].float().cpu()) < 5e-3


# ------------------------------------------------------------- attention ----


def _attn_reference(q, k, v, allow, nh, nkv, hd, do):
    """fp32 dense-mask attention with autograd (reference nn.py:84-88)."""
    S = q.shape[0]
    qf = q.float().cpu().view(S, nh, hd).transpose(0, 1).requires_grad_(True)
    kf = k.float().cpu().view(S, nkv, hd).transpose(0, 1).requires_grad_(True)
    vf = v.float().cpu().view(S, nkv, hd).transpose(0, 1).requires_grad_(True)
    rep = nh // nkv
    kk = kf.repeat_interleave(rep, 0)
    vv = vf.repeat_interleave(rep, 0)
    s = qf @ kk.transpose(-1, -2) / math.sqrt(hd)
    s = s.masked_fill(~allow, float("-inf"))
    o = torch.softmax(s, -1) @ vv
    o.backward(do.float().cpu().view(S, nh, hd).transpose(0, 1))
    flat = lambda t: t.transpose(0, 1).reshape(S, -1)  # noqa: E731
    return flat(o.detach()), flat(qf.grad), flat(kf.grad), flat(vf.grad)


def _partition_allow(a0, a1, k):
    anc, dep = oracle.segment_slots(a0, a1, k)
    return oracle.slot_allow(anc, dep)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("layout_kind", ["partition", "indexed", "bias"])
@pytest.mark.parametrize("geom", [(0, 9, 4, 4, 2, 8), (12, 40, 5, 4, 2, 64), (0, 33, 1, 2, 1, 128),
                                  (20, 70, 3, 28, 4, 128)])
def test_attention_simt_all_layouts(dtype, layout_kind, geom):
    a0, a1, k, nh, nkv, hd = geom
    allow = _partition_allow(a0, a1, k)
    S = allow.shape[0]
    q = _rand(S, nh * hd, dtype=dtype, seed=10)
    kt = _rand(S, nkv * hd, dtype=dtype, seed=11)
    vt = _rand(S, nkv * hd, dtype=dtype, seed=12)
    do = _rand(S, nh * hd, dtype=dtype, seed=13)
    if layout_kind == "partition":
        lay = ops.AttnLayout(L.LAYOUT_PARTITION, a0=a0, a1=a1, k=k)
    elif layout_kind == "indexed":
        anc, dep = oracle.segment_slots(a0, a1, k)
        lay = ops.AttnLayout(L.LAYOUT_INDEXED, anchor=anc.to(torch.int32).to(DEV),
                             depth=dep.to(torch.int32).to(DEV))
    else:
        bias = oracle.drafter_step.additive_bias(allow, dtype)[None, None].to(DEV)
        lay = ops.AttnLayout(L.LAYOUT_BIAS, bias=bias)
    o, lse = ops.attn_fwd(q[None], kt[None], vt[None], nh, nkv, hd, lay, algo=L.ALGO_SIMT)
    dq, dk, dv = ops.attn_bwd(q[None], kt[None], vt[None], o, do[None], lse, nh, nkv, hd, lay,
                              algo=L.ALGO_SIMT)
    torch.cuda.synchronize()
    ro, rdq, rdk, rdv = _attn_reference(q, kt, vt, allow, nh, nkv, hd, do)
    tol = 1e-5 if dtype == torch.float32 else 2e-2
    assert rel(o[0].float().cpu(), ro) < tol
    assert rel(dq[0].float().cpu(), rdq) < tol
    assert rel(dk[0].float().cpu(), rdk) < tol
    assert rel(dv[0].float().cpu(), rdv) < tol


TC_GEOMS = [(0, 300, 5, 4, 2), (256, 512, 5, 4, 1), (100, 333, 3, 8, 2), (0, 130, 1, 4, 2),
            (1500, 2048, 5, 2, 1), (0, 64, 8, 2, 2), (37, 41, 4, 4, 4),
            # 28 x 32 key-tile work items: several per CTA of the persistent dK/dV kernel
            (256, 1024, 5, 28, 4)]


def _qkv_view(S, nh, nkv, seed):
    """q/k/v as column blocks of one fused [S, (nh + 2 nkv) * 128] buffer, as the
    training step lays them out."""
    hd = 128
    cq, ckv = nh * hd, nkv * hd
    qkv = _rand(S, cq + 2 * ckv, seed=seed)
    v3 = qkv.view(1, S, -1)
    return v3[:, :, :cq], v3[:, :, cq:cq + ckv], v3[:, :, cq + ckv:]


@pytest.mark.parametrize("geom", TC_GEOMS)
def test_attention_tcgen05_fwd_matches_simt(geom):
    a0, a1, k, nh, nkv = geom
    S = a1 + (a1 - a0) * (k - 1)
    q, kt, vt = _qkv_view(S, nh, nkv, seed=30)
    lay = ops.AttnLayout(L.LAYOUT_PARTITION, a0=a0, a1=a1, k=k)
    o_ref, lse_ref = ops.attn_fwd(q, kt, vt, nh, nkv, 128, lay, algo=L.ALGO_SIMT)
    o, lse = ops.attn_fwd(q, kt, vt, nh, nkv, 128, lay, algo=L.ALGO_TCGEN05)
    torch.cuda.synchronize()
    ops.check_status(DEV)
    assert rel(o.float().cpu(), o_ref.float().cpu()) < 1e-2
    assert torch.allclose(lse.cpu(), lse_ref.cpu(), atol=2e-3, rtol=1e-4)


@pytest.mark.parametrize("variant", [0, 1, 2])
@pytest.mark.parametrize("geom", TC_GEOMS)
def test_attention_tcgen05_bwd_matches_simt(geom, variant):
    a0, a1, k, nh, nkv = geom
    S = a1 + (a1 - a0) * (k - 1)
    q, kt, vt = _qkv_view(S, nh, nkv, seed=31)
    do = _rand(1, S, nh * 128, seed=32)
    lay = ops.AttnLayout(L.LAYOUT_PARTITION, a0=a0, a1=a1, k=k)
    o, lse = ops.attn_fwd(q, kt, vt, nh, nkv, 128, lay, algo=L.ALGO_SIMT)
    ref = ops.attn_bwd(q, kt, vt, o, do, lse, nh, nkv, 128, lay, algo=L.ALGO_SIMT)
    # gradients written straight into a fused [S, q|k|v] buffer, as the training step does
    dqkv = torch.full((1, S, (nh + 2 * nkv) * 128), float("nan"), dtype=torch.bfloat16, device=DEV)
    cq, ckv = nh * 128, nkv * 128
    got = ops.attn_bwd(q, kt, vt, o, do, lse, nh, nkv, 128, lay, dq=dqkv[:, :, :cq],
                       dk=dqkv[:, :, cq:cq + ckv], dv=dqkv[:, :, cq + ckv:],
                       algo=L.ALGO_TCGEN05 | (variant << 8))
    torch.cuda.synchronize()
    ops.check_status(DEV)
    for name, a, b in zip(("dq", "dk", "dv"), got, ref):
        assert not torch.isnan(a).any(), name
        assert rel(a.float().cpu(), b.float().cpu()) < 2e-2, name


# (n, segments, K, Hq, Hkv): every segment of one sequence stacked in one row space
SEG_CASES = [(300, 4, 5, 4, 2), (2048, 4, 5, 28, 4), (100, 3, 1, 4, 2),
             # ten segments: two launch groups (at most eight segments per launch)
             (90, 10, 3, 2, 1), (700, 2, 8, 8, 2)]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("case", SEG_CASES)
def test_attention_segments_match_per_segment_calls(case, dtype):
    """One call over the stacked segments equals one call per segment: forward, lse
    and dQ bit for bit (the same tiles, only scheduled together); dK / dV up to the
    order of the fp32 GQA-group additions."""
    from parallel_eagle_b200.engine import segment_bounds

    n, nseg, k, nh, nkv = case
    if dtype == torch.float32 and n > 1000:
        pytest.skip("CUDA-core fp32 path: small cases only")
    hd = 128
    bounds = segment_bounds(n, nseg)
    rows = ops.segment_rows(bounds, k)
    R = sum(rows)
    cq, ckv = nh * hd, nkv * hd
    qkv = _rand(R, cq + 2 * ckv, dtype=dtype, seed=40)
    do = _rand(R, cq, dtype=dtype, seed=41)
    q, kt, vt = qkv[:, :cq], qkv[:, cq:cq + ckv], qkv[:, cq + ckv:]
    algo = L.ALGO_TCGEN05 if dtype == torch.bfloat16 else L.ALGO_SIMT
    o, lse = ops.attn_fwd_segments(q, kt, vt, nh, nkv, hd, bounds, k, algo=algo)
    dqkv = torch.full((R, cq + 2 * ckv), float("nan"), dtype=dtype, device=DEV)
    ops.attn_bwd_segments(q, kt, vt, o, do, lse, nh, nkv, hd, bounds, k, dq=dqkv[:, :cq],
                          dk=dqkv[:, cq:cq + ckv], dv=dqkv[:, cq + ckv:], algo=algo)
    off = 0
    for (a0, a1), S in zip(bounds, rows):
        lay = ops.AttnLayout(L.LAYOUT_PARTITION, a0=a0, a1=a1, k=k)
        sl = slice(off, off + S)
        o1, lse1 = ops.attn_fwd(q[None, sl], kt[None, sl], vt[None, sl], nh, nkv, hd, lay,
                                algo=algo)
        d1 = ops.attn_bwd(q[None, sl], kt[None, sl], vt[None, sl], o1, do[None, sl], lse1, nh,
                          nkv, hd, lay, algo=algo)
        torch.cuda.synchronize()
        ops.check_status(DEV)
        assert torch.equal(o[sl], o1[0]), (a0, a1)
        assert torch.equal(lse[nh * off : nh * (off + S)], lse1.reshape(-1)), (a0, a1)
        assert torch.equal(dqkv[sl, :cq], d1[0][0]), (a0, a1)
        for name, got, ref in (("dk", dqkv[sl, cq:cq + ckv], d1[1][0]),
                               ("dv", dqkv[sl, cq + ckv:], d1[2][0])):
            assert not torch.isnan(got).any(), name
            assert rel(got.float().cpu(), ref.float().cpu()) < 5e-3, (name, a0, a1)
        off += S


def test_attention_segments_reject_bad_rows():
    bounds = [(0, 64), (64, 128)]
    R = sum(ops.segment_rows(bounds, 3)) - 1
    q = torch.zeros(R, 256, dtype=torch.bfloat16, device=DEV)
    kv = torch.zeros(R, 128, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(L.PeError):
        ops.attn_fwd_segments(q, kv, kv, 2, 1, 128, bounds, 3)


# ----------------------------------------------------------- LM head + CE ----


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("soft", [False, True])
@pytest.mark.parametrize("R,H,V", [(37, 64, 1000), (130, 256, 20000), (700, 256, 40000)])
def test_lmhead_ce(dtype, soft, R, H, V):
    h = _rand(R, H, dtype=dtype, seed=14)
    W = _rand(V, H, dtype=dtype, seed=15, scale=0.05)
    labels = torch.randint(0, V, (R,), generator=torch.Generator().manual_seed(2)).to(DEV)
    teacher = _rand(R, H, dtype=dtype, seed=16) if soft else None
    loss = torch.zeros(1, dtype=torch.float32, device=DEV)
    scale = 0.37
    dh = ops.lmhead_ce(h, W, None if soft else labels, scale, loss, teacher=teacher)
    torch.cuda.synchronize()
    hr = h.float().cpu().requires_grad_(True)
    z = (hr @ W.float().cpu().t()).to(dtype).float()
    if soft:
        pt = torch.softmax((teacher.float().cpu() @ W.float().cpu().t()).to(dtype).float(), -1)
        lr = -(pt * torch.log_softmax(z, -1)).sum()
    else:
        lr = torch.nn.functional.cross_entropy(z, labels.cpu(), reduction="sum")
    (lr * scale).backward()
    assert abs(loss.item() - lr.item()) / abs(lr.item()) < 1e-4
    assert rel(dh.float().cpu(), hr.grad) < (1e-4 if dtype == torch.float32 else 2e-2)


@pytest.mark.parametrize("chunk_k", [0, 24, 32])
def test_lmhead_ce_full_vocab_against_torch(chunk_k):
    # the 7B-class head (vocab 152064) over a segment's worth of loss rows: the
    # fused one-GEMM path against torch's dense logits -> cross-entropy -> backward,
    # with the default 16K-column vocabulary chunks and with 24K / 32K ones (up to
    # 256 tile stats folded per row and chunk)
    R, H, V = 1100, 3584, 152064
    h = _rand(R, H, seed=40)
    W = _rand(V, H, seed=41, scale=0.02)
    labels = torch.randint(0, V, (R,), generator=torch.Generator().manual_seed(5)).to(DEV)
    loss = torch.zeros(1, dtype=torch.float32, device=DEV)
    scale = 1.0 / 3000
    dh = ops.lmhead_ce(h, W, labels, scale, loss, algo=L.ALGO_AUTO | (chunk_k << 8))
    ops.check_status(DEV)
    hr = h.detach().clone().requires_grad_(True)
    z = (hr @ W.t()).float()
    lr = torch.nn.functional.cross_entropy(z, labels, reduction="sum")
    (lr * scale).backward()
    torch.cuda.synchronize()
    assert abs(loss.item() - lr.item()) / lr.item() < 1e-4
    assert rel(dh.float(), hr.grad.float()) < 2e-2


@pytest.mark.parametrize("chunk_k,group_r,two_pass", [(1, 1, 0), (3, 2, 0), (0, 0, 0), (1, 1, 1),
                                                     (3, 2, 1)])
def test_lmhead_ce_row_groups_and_chunks(chunk_k, group_r, two_pass):
    # the fast path over several loss-row groups (ragged last group) and several
    # vocabulary chunks (ragged last chunk), with the later chunks one-pass (default)
    # or two-pass (algo bit 28): same loss and gradient as one pass
    R, H, V = 700, 256, 5000
    h = _rand(R, H, seed=42)
    W = _rand(V, H, seed=43, scale=0.05)
    labels = torch.randint(0, V, (R,), generator=torch.Generator().manual_seed(6))
    labels[5::7] = -100
    loss = torch.zeros(1, dtype=torch.float32, device=DEV)
    algo = L.ALGO_AUTO | (chunk_k << 8) | (group_r << 16) | (two_pass << 28)
    dh = ops.lmhead_ce(h, W, labels.to(DEV), 0.01, loss, algo=algo)
    torch.cuda.synchronize()
    ops.check_status(DEV)
    hr = h.float().cpu().requires_grad_(True)
    z = (hr @ W.float().cpu().t()).bfloat16().float()
    lr = torch.nn.functional.cross_entropy(z, labels, reduction="sum", ignore_index=-100)
    (lr * 0.01).backward()
    assert abs(loss.item() - lr.item()) / lr.item() < 1e-4
    assert rel(dh.float().cpu(), hr.grad) < 2e-2


@pytest.mark.parametrize("chunk_k", [0, 16, 8])
def test_lmhead_soft_targets_across_chunk_widths(chunk_k):
    """Soft-target loss over 40000 vocabulary rows in 32K (default; the 512-thread combine),
    16K or 8K chunks (the 256-thread one): same loss and gradient as dense fp32 torch."""
    R, H, V = 600, 256, 40000
    h = _rand(R, H, seed=45)
    W = _rand(V, H, seed=46, scale=0.05)
    teacher = _rand(R, H, seed=47)
    loss = torch.zeros(1, dtype=torch.float32, device=DEV)
    dh = ops.lmhead_ce(h, W, None, 0.5, loss, teacher=teacher, algo=L.ALGO_AUTO | (chunk_k << 8))
    torch.cuda.synchronize()
    ops.check_status(DEV)
    hr = h.float().cpu().requires_grad_(True)
    z = (hr @ W.float().cpu().t()).bfloat16().float()
    pt = torch.softmax((teacher.float().cpu() @ W.float().cpu().t()).bfloat16().float(), -1)
    lr = -(pt * torch.log_softmax(z, -1)).sum()
    (lr * 0.5).backward()
    assert abs(loss.item() - lr.item()) / abs(lr.item()) < 1e-4
    assert rel(dh.float().cpu(), hr.grad) < 2e-2


@pytest.mark.parametrize("boost", [40.0, 150.0])
@pytest.mark.parametrize("who", ["student", "teacher"])
def test_lmhead_soft_late_chunk_maximum(who, boost):
    """Soft targets with a late-chunk maximum in the student's or the teacher's logits:
    carried by the folds' rescale factors (~40 above the first chunk's maximum) or, past
    e^64 (~150), by the two-pass recomputation.  Against dense fp32 torch."""
    R, H, V = 600, 256, 5000
    g = torch.Generator().manual_seed(48)
    u = torch.randn(H, generator=g)
    u = u / u.norm()
    h = torch.randn(R, H, generator=g)
    tch = torch.randn(R, H, generator=g)
    big = torch.arange(0, R, 3)
    (h if who == "student" else tch)[big] += (boost / 1.5) * u
    W = torch.randn(V, H, generator=g) * 0.05
    W[3500] = 1.5 * u
    h, tch, W = h.bfloat16(), tch.bfloat16(), W.bfloat16()
    loss = torch.zeros(1, dtype=torch.float32, device=DEV)
    dh = ops.lmhead_ce(h.to(DEV), W.to(DEV), None, 0.01, loss, teacher=tch.to(DEV),
                       algo=L.ALGO_AUTO | (1 << 8))  # 1024-column chunks: five chunks
    torch.cuda.synchronize()
    ops.check_status(DEV)
    hr = h.float().requires_grad_(True)
    z = (hr @ W.float().t()).bfloat16().float()
    pt = torch.softmax((tch.float() @ W.float().t()).bfloat16().float(), -1)
    lr = -(pt * torch.log_softmax(z, -1)).sum()
    (lr * 0.01).backward()
    assert torch.isfinite(dh.float()).all()
    assert abs(loss.item() - lr.item()) / abs(lr.item()) < 1e-4
    assert rel(dh.float().cpu(), hr.grad) < 2e-2


@pytest.mark.parametrize("boost", [40.0, 150.0])
def test_lmhead_ce_late_chunk_maximum(boost):
    """Rows whose largest logit lies in a late vocabulary chunk, far above the first
    chunk's maximum.  Every chunk after the first writes e^(z - running max) straight
    from the logits GEMM; a jump of ~40 is carried by the fold's rescale factors, one of
    ~150 (beyond e^64) sets the overflow word and the classic two-pass recomputation
    runs instead.  Loss and gradient against fp32 torch either way."""
    R, H, V = 600, 256, 5000
    g = torch.Generator().manual_seed(44)
    u = torch.randn(H, generator=g)
    u = u / u.norm()
    h = torch.randn(R, H, generator=g)
    big = torch.arange(0, R, 3)
    h[big] += (boost / 1.5) * u  # logit ~ boost at column 3500 for every third row
    W = torch.randn(V, H, generator=g) * 0.05
    W[3500] = 1.5 * u
    h, W = h.bfloat16(), W.bfloat16()
    labels = torch.randint(0, V, (R,), generator=g)
    labels[big[::2]] = 3500
    labels[7::11] = -100
    loss = torch.zeros(1, dtype=torch.float32, device=DEV)
    dh = ops.lmhead_ce(h.to(DEV), W.to(DEV), labels.to(DEV), 0.01, loss,
                       algo=L.ALGO_AUTO | (1 << 8))  # 1024-column chunks: five chunks
    torch.cuda.synchronize()
    ops.check_status(DEV)
    hr = h.float().requires_grad_(True)
    z = (hr @ W.float().t()).bfloat16().float()
    assert (z[big].max(1).values - z[big, :1024].max(1).values).min() > boost * 0.6
    lr = torch.nn.functional.cross_entropy(z, labels, reduction="sum", ignore_index=-100)
    (lr * 0.01).backward()
    assert torch.isfinite(dh.float()).all()
    assert abs(loss.item() - lr.item()) / lr.item() < 1e-4
    assert rel(dh.float().cpu(), hr.grad) < 2e-2


@pytest.mark.parametrize("V", [300, 304])
def test_lmhead_ignores_negative_labels(V):
    R, H = 20, 64
    h = _rand(R, H, seed=17)
    W = _rand(V, H, seed=18, scale=0.05)
    labels = torch.randint(0, V, (R,), generator=torch.Generator().manual_seed(3))
    labels[::3] = -100
    loss = torch.zeros(1, dtype=torch.float32, device=DEV)
    dh = ops.lmhead_ce(h, W, labels.to(DEV), 1.0, loss)
    torch.cuda.synchronize()
    assert torch.all(dh[::3].float() == 0)
    keep = labels >= 0
    z = (h.float().cpu()[keep] @ W.float().cpu().t()).bfloat16().float()
    ref = torch.nn.functional.cross_entropy(z, labels[keep], reduction="sum")
    assert abs(loss.item() - ref.item()) / ref.item() < 1e-4


# ------------------------------------------------------------- small ops ----


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_swiglu_fwd_bwd(dtype):
    rows, inter = 33, 96
    gu = _rand(rows, 2 * inter, dtype=dtype, seed=19)
    da = _rand(rows, inter, dtype=dtype, seed=20)
    a = ops.swiglu_fwd(gu, inter)
    dgu = ops.swiglu_bwd(da, gu, inter)
    torch.cuda.synchronize()
    g = gu.float().cpu().requires_grad_(True)
    ref = torch.nn.functional.silu(g[:, :inter]) * g[:, inter:]
    ref.backward(da.float().cpu())
    tol = 1e-6 if dtype == torch.float32 else 2e-2
    assert rel(a.float().cpu(), ref.detach()) < tol
    assert rel(dgu.float().cpu(), g.grad) < tol


# H 40 (bf16 rows of 80 B): element-wise kernels; H 3584 / fp32 H 64: 16-byte row moves
@pytest.mark.parametrize("H,dtype", [(40, torch.bfloat16), (3584, torch.bfloat16),
                                     (64, torch.float32)])
def test_rows_embed_fill_gather_scatter_colsum(H, dtype):
    E = _rand(50, H, seed=21, dtype=dtype)
    ids = torch.tensor([3, 0, 49, 3], device=DEV)
    out = torch.zeros(4, 2 * H, dtype=dtype, device=DEV)
    ops.embed_rows(ids, E, out[:, :H])
    assert torch.equal(out[:, :H], E[ids]) and torch.all(out[:, H:] == 0)
    vec = _rand(H, seed=22, dtype=dtype)
    dst = torch.zeros(5, H, dtype=dtype, device=DEV)
    ops.fill_rows(vec, dst[1:4])
    assert torch.equal(dst[1:4], vec.expand(3, H)) and torch.all(dst[0] == 0)
    src = _rand(6, H, seed=23, dtype=dtype)
    idx = torch.tensor([5, 1, 2], device=DEV)
    g = ops.gather_rows(src, idx)
    assert torch.equal(g, src[idx])
    back = torch.zeros_like(src)
    ops.scatter_rows(g, idx, back)
    assert torch.equal(back[idx], src[idx]) and torch.all(back[0] == 0)
    s = ops.rowsum_cols(src)
    assert rel(s.cpu(), src.float().sum(0).cpu()) < 1e-6


@pytest.mark.parametrize("dtype,H,ldx", [(torch.bfloat16, 3584, 3584), (torch.float32, 1000, 1000),
                                         (torch.bfloat16, 300, 300), (torch.bfloat16, 256, 264)])
def test_rowsum_cols_ranges(dtype, H, ldx):
    """Column sums over several row ranges in one launch (the clustered 16-byte kernel,
    or per range on the scalar one when H is not a multiple of 8): the segments'
    prediction rows of a stacked pass, an empty and a one-row range, and more than 16
    ranges (two launches), against fp64 sums."""
    rows = 9000
    xs = _rand(rows, ldx, seed=25, dtype=dtype)
    x = xs[:, :H]
    cases = [[(2560, 4608), (7680, 9000)], [(0, 0), (5, 6), (100, 3000)],
             [(i * 400, i * 400 + 37 * (i + 1)) for i in range(20)]]
    for ranges in cases:
        got = ops.rowsum_cols_ranges(x, ranges)
        torch.cuda.synchronize()
        want = sum(x[b:e].double().sum(0) for b, e in ranges).cpu()
        err = (got.double().cpu() - want).abs().max().item()
        assert err <= 1e-4 * (1.0 + want.abs().max().item()), (ranges[:3], err)
    with pytest.raises(L.PeError):
        ops.rowsum_cols_ranges(x, [(5, rows + 1)])


def test_row_moves_beyond_one_grid_row_span():
    """More rows than the 16-byte row kernel's grid covers in one pass (32768)."""
    src = _rand(1000, 64, seed=24)
    idx = torch.randint(0, 1000, (40000,), generator=torch.Generator().manual_seed(3)).to(DEV)
    g = ops.gather_rows(src, idx)
    assert torch.equal(g, src[idx])
    dst = torch.zeros(40000, 64, dtype=torch.bfloat16, device=DEV)
    ops.fill_rows(src[7], dst)
    assert torch.equal(dst, src[7].expand(40000, 64))


def test_adamw_with_clipping_matches_torch():
    n = 5000
    g = torch.Generator().manual_seed(4)
    p0 = torch.randn(n, generator=g)
    grads = [torch.randn(n, generator=g) * 3 for _ in range(3)]
    p_ref = p0.clone().requires_grad_(True)
    opt = torch.optim.AdamW([p_ref], lr=1e-2, weight_decay=0.1)
    p = p0.clone().to(DEV)
    m = torch.zeros(n, device=DEV)
    v = torch.zeros(n, device=DEV)
    for step, gr in enumerate(grads, 1):
        p_ref.grad = gr.clone()
        torch.nn.utils.clip_grad_norm_([p_ref], 1.0)
        opt.step()
        gd = gr.to(DEV)
        ss = torch.zeros(1, device=DEV)
        ops.sumsq_into(gd, ss)
        ops.adamw_step(p, gd, m, v, ss, 1.0, 1e-2, 0.9, 0.999, 1e-8, 0.1, step)
    torch.cuda.synchronize()
    assert rel(p.cpu(), p_ref.detach()) < 1e-5


def test_sumsq_is_deterministic_and_exact():
    """The global-norm reduction behind the clip (``ops.sumsq_into``): the same gradient
    gives the same bits on every call -- as every data-parallel rank must, or the
    replicas' clip coefficients and updates drift apart -- and matches an fp64 sum."""
    g = _rand(40_000_003, dtype=torch.bfloat16, seed=90, scale=0.01)
    outs = []
    for _ in range(3):
        out = torch.zeros(1, dtype=torch.float32, device=DEV)
        ops.sumsq_into(g, out)
        outs.append(out.clone())
    torch.cuda.synchronize()
    assert all(torch.equal(outs[0], o) for o in outs[1:])
    ref = g.double().pow(2).sum().item()
    assert abs(outs[0].item() - ref) / ref < 1e-5
    # accumulates into the existing value
    acc = torch.full((1,), 2.5, dtype=torch.float32, device=DEV)
    ops.sumsq_into(g, acc)
    assert abs(acc.item() - (2.5 + ref)) / ref < 1e-5


@pytest.mark.parametrize("src_dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("H,n,mapped", [(256, 50, False), (3584, 300, True), (512, 97, True)])
def test_feature_norm_matches_cast_gather_rmsnorm(src_dtype, dtype, H, n, mapped):
    """The fused ingestion norm (reference drafter.py:129-130) against the unfused
    sequence -- cast the shard to the run dtype, gather the mapped token rows, RMSNorm
    the H-wide blocks -- and its weight gradient against the RMSNorm backward's dW.
    The row's sum of squares is reduced in a different order (8 columns per thread
    across the block, against strided 16-byte chunks in one warp), so rstd agrees to
    fp32 rounding (2e-6 relative); y = x rstd w then agrees to that plus two roundings
    in fp32, and to one unit in the last place in bf16, where a flip is rare."""
    nfl = 3
    g = torch.Generator().manual_seed(H + n)
    feats = (torch.randn(n, nfl * H, generator=g) * 2).to(src_dtype).to(DEV)
    w = (1 + 0.1 * torch.randn(H, generator=g)).to(dtype).to(DEV)
    if mapped:  # a stacked pass's real rows: prefixes of two segments
        tok = torch.cat([torch.arange(n // 2), torch.arange(n)]).to(DEV)
    else:
        tok = None
    T = n + n // 2 if mapped else n
    y, rstd = ops.feature_norm_fwd(feats, w, nfl, H, dtype, 1e-5, src_tok=tok, tokens=T)
    src = feats.to(dtype)
    rows = ops.gather_rows(src, tok) if mapped else src
    ref, ref_rstd = ops.rmsnorm_fwd(rows.reshape(T * nfl, H), w, 1e-5)
    torch.cuda.synchronize()
    assert torch.allclose(rstd, ref_rstd, rtol=2e-6, atol=0)
    tol = 2.0 ** -7 if dtype == torch.bfloat16 else 2e-6 + 2.0 ** -22
    diff = (y.float() - ref.float()).abs()
    assert torch.all(diff <= tol * ref.float().abs().clamp_min(1e-30)), diff.max()
    if dtype == torch.bfloat16:
        assert (diff > 0).float().mean().item() < 0.02  # only rare rounding flips
    dy = (torch.randn(T * nfl, H, generator=g)).to(dtype).to(DEV)
    part = ops.feature_norm_dw(dy, feats, rstd, nfl, H, src_tok=tok)
    dw = ops.colsum_into(part, torch.zeros(H, dtype=torch.float32, device=DEV), accumulate=False)
    _, rpart = ops.rmsnorm_bwd(dy, rows.reshape(T * nfl, H), w, ref_rstd)
    rdw = ops.colsum_into(rpart, torch.zeros(H, dtype=torch.float32, device=DEV), accumulate=False)
    torch.cuda.synchronize()
    assert rel(dw.cpu(), rdw.cpu()) < 1e-5
