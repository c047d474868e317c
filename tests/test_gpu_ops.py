"""Per-kernel numerics on the GPU against plain torch fp32 references (through the C-ABI)."""
import ctypes

import pytest
import torch
import torch.nn.functional as F

from tt_atom import _lib as L
from tt_atom._lib import call, ptr

pytestmark = pytest.mark.gpu
dev = "cuda"


def s():
    return L.stream_ptr()


def rnd(*shape, seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return torch.randn(*shape, generator=g).to(dev)


def close(a, b, tol=1e-5):
    a, b = a.double(), b.double()
    err = (a - b).abs().max().item()
    scale = max(b.abs().max().item(), 1.0)
    assert err <= tol * scale, f"max err {err} (scale {scale})"


# ------------------------------------------------------------------- reference-op equivalents

def _pattern():
    # the uma-s 9x9 block-diagonal pattern, grouped by output row (tt_atom/rotation.py:145-165)
    ij = [(i, j) for i in range(9) for j in range(9)
          if (i == 0 and j == 0) or (1 <= i < 4 and 1 <= j < 4) or (i >= 4 and j >= 4)]
    return ij


def test_fused_rotate_and_gc():
    ij = _pattern()
    nnz, E, W = len(ij), 1000, 256
    x, coef, gout = rnd(E, 9 * W), rnd(E, nnz, seed=1), rnd(E, 9 * W, seed=2)
    deg = [sum(1 for (i, j) in ij if i == b) for b in range(9)]
    ks = [k for b in range(9) for k, (i, j) in enumerate(ij) if i == b]
    js = [ij[k][1] for k in ks]
    out = torch.empty(E, 9 * W, device=dev)
    call("atom_fused_rotate", ptr(x), ptr(coef), E, 9, 9, W, nnz, L.host_i32(deg), L.host_i32(ks),
         L.host_i32(js), ptr(out), s())
    Wd = torch.zeros(E, 9, 9, device=dev)
    for k, (i, j) in enumerate(ij):
        Wd[:, i, j] = coef[:, k]
    ref = torch.bmm(Wd, x.view(E, 9, W)).reshape(E, -1)
    close(out, ref)
    gc = torch.empty(E, nnz, device=dev)
    call("atom_fused_rotate_gc", ptr(gout), ptr(x), E, 9, 9, W, nnz,
         L.host_i32([i for i, j in ij]), L.host_i32([j for i, j in ij]), ptr(gc), s())
    g3, x3 = gout.view(E, 9, W), x.view(E, 9, W)
    ref = torch.stack([(g3[:, i] * x3[:, j]).sum(-1) for i, j in ij], 1)
    close(gc, ref, 1e-5)


def test_fused_gate_and_ln_bw():
    E, H, G = 513, 32, 256
    a, gate, b = rnd(E, H + G), rnd(E, G, seed=1), rnd(E, H + G, seed=2)
    out = torch.empty_like(a)
    call("atom_fused_gate", ptr(a), ptr(gate), ptr(b), E, H, G, 0, ptr(out), s())
    close(out, torch.cat([F.silu(a[:, :H]), a[:, H:] * gate], 1))
    call("atom_fused_gate", ptr(a), ptr(gate), ptr(b), E, H, G, 1, ptr(out), s())
    sb = torch.sigmoid(b[:, :H])
    close(out, torch.cat([a[:, :H] * sb * (1 + b[:, :H] * (1 - sb)), a[:, H:] * gate], 1))
    W = 128
    x = rnd(E, W).requires_grad_()
    gamma, beta, g = rnd(W, seed=3), rnd(W, seed=4), rnd(E, W, seed=5)
    n = F.layer_norm(x, (W,), gamma, beta, 1e-5)
    y = F.silu(n)
    (ref,) = torch.autograd.grad(y, x, g)
    dx = torch.empty(E, W, device=dev)
    call("atom_fused_ln_bw", ptr(g), ptr(x.detach()), ptr(n.detach()), ptr(gamma), E, W, 1e-5,
         ptr(dx), s())
    close(dx, ref, 1e-4)


# ------------------------------------------------------------------------------- GEMM

TOL = {0: 1e-5, 1: 5e-3, 2: 1e-5, 3: 1e-5}


def gemm(A, lda, M, groups, C, ldc, Cpre, T1, T2, i1, i2, ldt, act, acc, precision):
    """atom_gemm_ex with a scratch large enough for the fp16-pair mode's row scales (and
    split-K partials); other modes get no scratch (plain atom_gemm)."""
    sc = None
    if precision == 3:
        groups.ensure_f16()
        sc = torch.empty(8 * ((M + 127) // 128 * 128) * max(ldc, 64) + 1024, device=dev)
    call("atom_gemm_ex", ptr(A), lda, M, ctypes.byref(groups.struct), ptr(C), ldc, ptr(Cpre),
         ptr(T1), ptr(T2), ptr(i1), ptr(i2), ldt, act, acc, precision, ptr(sc),
         sc.numel() if sc is not None else 0, s())


@pytest.mark.parametrize("precision", [0, 1, 2, 3])
@pytest.mark.parametrize("M", [1, 129, 1000])
@pytest.mark.parametrize("N2", [130, 132])
def test_grouped_gemm_with_epilogues(M, precision, N2):
    """Bias, two gathered node tables, SiLU with the pre-activation kept, then accumulate.
    N2 = 132 keeps every group a multiple of 4 columns (tensor-core launches then take the
    TMA-store epilogue, tables added per row); N2 = 130 takes the row-store epilogue."""
    from tt_atom.engine import _Groups
    K1, N1, K2 = 96, 160, 64
    A = rnd(M, K1 + K2)
    B1, B2 = rnd(K1, N1, seed=1), rnd(K2, N2, seed=2)
    bias1 = rnd(N1, seed=3)
    T1, T2 = rnd(10, 400, seed=4), rnd(10, 400, seed=5)
    i1 = torch.randint(0, 10, (M,), device=dev, dtype=torch.int32)
    i2 = torch.randint(0, 10, (M,), device=dev, dtype=torch.int32)
    g = _Groups([dict(a_col=0, K=K1, c_col=0, N=N1, B=B1, bias=bias1, t_col=0),
                 dict(a_col=K1, K=K2, c_col=N1, N=N2, B=B2, t_col=200)])
    C = torch.empty(M, N1 + N2, device=dev)
    Cpre = torch.empty(M, N1 + N2, device=dev)
    gemm(A, K1 + K2, M, g, C, N1 + N2, Cpre, T1, T2, i1, i2, 400, 1, 0, precision)
    Ad = A.double()
    r1 = Ad[:, :K1] @ B1.double() + bias1.double() + T1.double()[i1.long(), :N1] + \
        T2.double()[i2.long(), :N1]
    r2 = Ad[:, K1:] @ B2.double() + T1.double()[i1.long(), 200:200 + N2] + \
        T2.double()[i2.long(), 200:200 + N2]
    pre = torch.cat([r1, r2], 1)
    close(Cpre, pre, TOL[precision])
    close(C, F.silu(pre), TOL[precision])
    # accumulate
    C2 = C.clone()
    gemm(A, K1 + K2, M, g, C2, N1 + N2, None, T1, T2, i1, i2, 400, 0, 1, precision)
    close(C2, C.double() + pre, TOL[precision])
    code = ctypes.c_int(-1)
    call("atom_device_error", ctypes.byref(code), s())
    assert code.value == 0


@pytest.mark.parametrize("precision", [1, 2, 3])
@pytest.mark.parametrize("M", [1, 129, 1000])
@pytest.mark.parametrize("N2", [132, 130])
def test_gemm_tma_store_epilogue(M, precision, N2):
    """Launches without gathered tables take the TMA-store epilogue: bias + SiLU with the
    pre-activation kept, then an accumulating launch (TMA reduce-add); N2 = 132 and the row
    counts leave ragged tile edges that the tensor maps must clip. N2 = 130 (not a multiple of
    4 columns) takes the row-store path instead; both must leave the columns around the groups
    untouched."""
    from tt_atom.engine import _Groups
    K1, N1, K2 = 96, 160, 64
    A = rnd(M, K1 + K2)
    B1, B2 = rnd(K1, N1, seed=1), rnd(K2, N2, seed=2)
    bias1 = rnd(N1, seed=3)
    g = _Groups([dict(a_col=0, K=K1, c_col=0, N=N1, B=B1, bias=bias1),
                 dict(a_col=K1, K=K2, c_col=N1 + 4, N=N2, B=B2)])
    ldc = N1 + 4 + N2 + 2
    C = torch.full((M, ldc), 7.0, device=dev)
    Cpre = torch.full((M, ldc), 7.0, device=dev)
    gemm(A, K1 + K2, M, g, C, ldc, Cpre, None, None, None, None, 0, 1, 0, precision)
    Ad = A.double()
    pre = torch.cat([Ad[:, :K1] @ B1.double() + bias1.double(), Ad[:, K1:] @ B2.double()], 1)
    cols = torch.cat([torch.arange(N1), torch.arange(N1 + 4, N1 + 4 + N2)]).to(dev)
    close(Cpre[:, cols], pre, TOL[precision])
    close(C[:, cols], F.silu(pre), TOL[precision])
    gap = torch.ones(ldc, dtype=torch.bool, device=dev)
    gap[cols] = False
    assert (C[:, gap] == 7.0).all() and (Cpre[:, gap] == 7.0).all()   # nothing outside the groups
    C2 = C.clone()
    gemm(A, K1 + K2, M, g, C2, ldc, None, None, None, None, None, 0, 0, 1, precision)
    close(C2[:, cols], C[:, cols].double() + pre, TOL[precision])
    assert (C2[:, gap] == 7.0).all()


@pytest.mark.parametrize("precision", [1, 2, 3])
@pytest.mark.parametrize("M", [100, 1002])
def test_gemm_split_k_with_scratch(M, precision):
    """atom_gemm_ex with a scratch buffer: a launch with few row tiles splits K over more CTAs,
    writes raw partial products to the scratch and sums them in a fixed order, then applies
    bias, SiLU, the kept pre-activation and accumulation. Results match float64 within the
    precision's tolerance, are bit-identical run to run, leave the columns around the groups
    untouched, and a scratch too small to split gives the unsplit answer."""
    from tt_atom.engine import _Groups
    K1, N1, K2, N2 = 1024, 384, 512, 256
    A = rnd(M, K1 + K2) * 0.1
    B1, B2 = rnd(K1, N1, seed=1) * 0.1, rnd(K2, N2, seed=2) * 0.1
    bias1, bias2 = rnd(N1, seed=3), rnd(N2, seed=4)
    g = _Groups([dict(a_col=0, K=K1, c_col=0, N=N1, B=B1, bias=bias1),
                 dict(a_col=K1, K=K2, c_col=N1 + 4, N=N2, B=B2, bias=bias2)]).ensure_f16()
    ldc = N1 + 4 + N2 + 4
    mpad = (M + 127) // 128 * 128
    scratch = torch.empty(8 * mpad * ldc, device=dev)

    def run(sc, n_sc, act=1, acc=0, C0=None):
        C = torch.full((M, ldc), 7.0, device=dev) if C0 is None else C0.clone()
        Cpre = torch.full((M, ldc), 7.0, device=dev)
        call("atom_gemm_ex", ptr(A), K1 + K2, M, ctypes.byref(g.struct), ptr(C), ldc,
             ptr(Cpre) if act else None, None, None, None, None, 0, act, acc, precision,
             ptr(sc), n_sc, s())
        return C, Cpre

    Ad = A.double()
    pre = torch.cat([Ad[:, :K1] @ B1.double() + bias1.double(),
                     Ad[:, K1:] @ B2.double() + bias2.double()], 1)
    cols = torch.cat([torch.arange(N1), torch.arange(N1 + 4, N1 + 4 + N2)]).to(dev)
    gap = torch.ones(ldc, dtype=torch.bool, device=dev)
    gap[cols] = False
    C, Cpre = run(scratch, scratch.numel())
    close(Cpre[:, cols], pre, TOL[precision])
    close(C[:, cols], F.silu(pre), TOL[precision])
    assert (C[:, gap] == 7.0).all() and (Cpre[:, gap] == 7.0).all()
    C_again, _ = run(scratch, scratch.numel())
    assert torch.equal(C, C_again)
    C_small, _ = run(scratch, 1024)             # too small to split: the unsplit launch
    close(C_small[:, cols], F.silu(pre), TOL[precision])
    C_acc, _ = run(scratch, scratch.numel(), act=0, acc=1, C0=C)
    close(C_acc[:, cols], C[:, cols].double() + pre, TOL[precision])
    assert (C_acc[:, gap] == 7.0).all()


def test_gemm_3xtf32_split_is_exact_for_truncating_tensor_cores():
    """3xTF32 leaves A in shared memory as loaded and relies on the tensor core reading an fp32
    operand as TF32 by dropping its low 13 mantissa bits (truncation); A_lo = A - trunc(A) is
    exact. A = 1 + 3 * 2^-12 lies 0.75 TF32 ulp above 1: truncation gives 1 and the product
    with B = 1 comes out exact; a rounding tensor core would give 1 + 2^-10 + 3 * 2^-12."""
    from tt_atom.engine import _Groups
    M, K, N = 128, 32, 32
    A = torch.zeros(M, K, device=dev)
    A[:, 0] = 1.0 + 3.0 * 2.0 ** -12
    B = torch.zeros(K, N, device=dev)
    B[0, :] = 1.0
    g = _Groups([dict(a_col=0, K=K, c_col=0, N=N, B=B)])
    C = torch.empty(M, N, device=dev)
    call("atom_gemm", ptr(A), K, M, ctypes.byref(g.struct), ptr(C), N, None, None, None, None,
         None, 0, 0, 0, 2, s())
    assert (C == 1.0 + 3.0 * 2.0 ** -12).all()


@pytest.mark.parametrize("precision", [1, 2, 3])
def test_tensor_core_gemm_so2_shapes_many_groups(precision):
    """The so2_conv_1 block layout (K = 768, 1024, 512) and an 8-group radial-style layout."""
    from tt_atom.engine import _Groups
    M = 3001
    A = rnd(M, 2304)
    Bs = [rnd(768, 640, seed=1) * 0.05, rnd(1024, 512, seed=2) * 0.05, rnd(512, 256, seed=3) * 0.05]
    bias0 = rnd(640, seed=4)
    g = _Groups([dict(a_col=0, K=768, c_col=0, N=640, B=Bs[0], bias=bias0),
                 dict(a_col=768, K=1024, c_col=640, N=512, B=Bs[1]),
                 dict(a_col=1792, K=512, c_col=1152, N=256, B=Bs[2])])
    C = torch.empty(M, 1408, device=dev)
    gemm(A, 2304, M, g, C, 1408, None, None, None, None, None, 0, 0, 0, precision)
    Ad = A.double()
    ref = torch.cat([Ad[:, :768] @ Bs[0].double() + bias0.double(),
                     Ad[:, 768:1792] @ Bs[1].double(), Ad[:, 1792:] @ Bs[2].double()], 1)
    close(C, ref, TOL[precision])
    G, EC = 8, 32
    X = rnd(M, G * EC, seed=9)
    Ws = [rnd(EC, EC + 8 * k, seed=10 + k) for k in range(G)]
    offs = [0]
    for w_ in Ws:
        offs.append(offs[-1] + w_.shape[1])
    g = _Groups([dict(a_col=k * EC, K=EC, c_col=offs[k], N=Ws[k].shape[1], B=Ws[k])
                 for k in range(G)])
    C = torch.empty(M, offs[-1], device=dev)
    gemm(X, G * EC, M, g, C, offs[-1], None, None, None, None, None, 0, 0, 0, precision)
    ref = torch.cat([X[:, k * EC:(k + 1) * EC].double() @ Ws[k].double() for k in range(G)], 1)
    close(C, ref, TOL[precision])


def test_gemm_f16_pair_exact_on_small_integers():
    """Known answer for the fp16-pair mode's operand layout (two fp16 per tensor-memory column,
    64-byte swizzled weights): small integers are exact in every split, so C must equal the
    integer product exactly, for every row, column and K position."""
    from tt_atom.engine import _Groups
    M, K, N = 256, 96, 160
    g0 = torch.Generator(device="cpu").manual_seed(5)
    A = torch.randint(-8, 9, (M, K), generator=g0).float().to(dev)
    B = torch.randint(-8, 9, (K, N), generator=g0).float().to(dev)
    g = _Groups([dict(a_col=0, K=K, c_col=0, N=N, B=B)])
    C = torch.empty(M, N, device=dev)
    gemm(A, K, M, g, C, N, None, None, None, None, None, 0, 0, 0, 3)
    assert torch.equal(C, (A.double() @ B.double()).float())


def test_gemm_f16_pair_wide_magnitude_range():
    """fp16 covers only ~2^-24 .. 2^16, so the fp16-pair mode scales every A row (per group)
    and every B column by a power of two. Rows over 1e-15 .. 1e15 and columns over
    1e-10 .. 1e10 (products stay inside fp32), an all-zero row and a row with one entry 1e9
    times the others must still come out with fp32-level error relative to sum |a| |b|."""
    from tt_atom.engine import _Groups
    M, K, N = 300, 256, 192
    A = rnd(M, K, seed=21)
    g0 = torch.Generator(device="cpu").manual_seed(23)
    rs = torch.logspace(-15, 15, M)[torch.randperm(M, generator=g0)].to(dev)
    A = A * rs[:, None]
    A[7] = 0.0
    A[11] = A[11] / A[11].abs().max() * 1e-3
    A[11, 5] = 1.0e6                     # one dominant entry in an otherwise small row
    B = rnd(K, N, seed=22) * torch.logspace(-10, 10, N, device=dev)[None, :]
    g = _Groups([dict(a_col=0, K=K, c_col=0, N=N, B=B)])
    C = torch.empty(M, N, device=dev)
    gemm(A, K, M, g, C, N, None, None, None, None, None, 0, 0, 0, 3)
    Ad, Bd = A.double(), B.double()
    ref = Ad @ Bd
    bound = (Ad.abs() @ Bd.abs())              # sum_k |a_mk| |b_kn|
    err = (C.double() - ref).abs()
    assert torch.isfinite(C).all()
    assert (err <= 2e-6 * bound + 1e-300).all(), float((err / (bound + 1e-300)).max())
    assert (C[7] == 0).all()


def test_gemm_f16_pair_without_scratch_runs_as_3xtf32():
    """Mode 3 needs a scratch for its row scales; without one (plain atom_gemm) the launch
    runs as 3xTF32 and gives exactly mode 2's result."""
    from tt_atom.engine import _Groups
    M, K, N = 500, 128, 192
    A, B = rnd(M, K, seed=31), rnd(K, N, seed=32)
    g = _Groups([dict(a_col=0, K=K, c_col=0, N=N, B=B)]).ensure_f16()
    C2, C3 = torch.empty(M, N, device=dev), torch.empty(M, N, device=dev)
    call("atom_gemm", ptr(A), K, M, ctypes.byref(g.struct), ptr(C2), N, None, None, None, None,
         None, 0, 0, 0, 2, s())
    call("atom_gemm", ptr(A), K, M, ctypes.byref(g.struct), ptr(C3), N, None, None, None, None,
         None, 0, 0, 0, 3, s())
    assert torch.equal(C2, C3)


def test_library_counts_its_launches():
    """atom_launch_count advances by the kernels one call launches: a mode-3 GEMM launches its
    row-scale pass and the GEMM."""
    from tt_atom.engine import _Groups, launch_count
    M, K, N = 500, 128, 192
    A, B = rnd(M, K, seed=31), rnd(K, N, seed=32)
    g = _Groups([dict(a_col=0, K=K, c_col=0, N=N, B=B)])
    C = torch.empty(M, N, device=dev)
    n0 = launch_count()
    gemm(A, K, M, g, C, N, None, None, None, None, None, 0, 0, 0, 3)
    assert launch_count() - n0 == 2
    n0 = launch_count()
    gemm(A, K, M, g, C, N, None, None, None, None, None, 0, 0, 0, 2)
    assert launch_count() - n0 == 1


# --------------------------------------------------------------------- node-side kernels

def _rms_ref(x, aw, ab, add0=None, eps=1e-5):
    lc = [0, 1, 1, 1, 2, 2, 2, 2, 2]
    bdw = torch.tensor([1.0 / (2 * l + 1) / 3 for l in lc], device=x.device).view(1, 9, 1)
    l0 = x[:, :1]
    xc = torch.cat([l0 - l0.mean(2, keepdim=True), x[:, 1:]], 1)
    fn = torch.rsqrt((xc * xc * bdw).sum(1, keepdim=True).mean(2, keepdim=True) + eps)
    out = xc * fn * aw[torch.tensor(lc, device=x.device)][None]
    b0 = ab.view(1, 1, -1) if add0 is None else ab.view(1, 1, -1) + add0[:, None, :]
    return torch.cat([out[:, :1] + b0, out[:, 1:]], 1)


@pytest.mark.parametrize("C", [16, 128])
def test_rmsnorm_sh_fwd_bwd(C):
    N = 300
    x = rnd(N, 9, C).requires_grad_()
    aw, ab, add0 = 1 + 0.1 * rnd(3, C, seed=1), rnd(C, seed=2), rnd(N, C, seed=3)
    g = rnd(N, 9, C, seed=4)
    ref = _rms_ref(x, aw, ab, add0)
    (gref,) = torch.autograd.grad(ref, x, g)
    out = torch.empty(N, 9, C, device=dev)
    call("atom_rmsnorm_sh_fwd", ptr(x.detach()), N, C, ptr(aw), ptr(ab), ptr(add0), 1e-5,
         ptr(out), s())
    close(out, ref, 1e-5)
    gx = torch.ones(N, 9, C, device=dev)
    call("atom_rmsnorm_sh_bwd", ptr(x.detach()), ptr(g), N, C, ptr(aw), 1e-5, 1, ptr(gx), s())
    close(gx, gref + 1, 1e-4)


@pytest.mark.parametrize("W", [32, 128, 256])
def test_ln_silu_groups_and_projection(W):
    """W = 32 takes the general warp loop, W = 128 / 256 the register-resident float4 forms
    (the backward also in place, dX aliasing gY)."""
    E, G = 777, 5
    X = rnd(E, G * W).requires_grad_()
    gam, bet, gY = 1 + 0.1 * rnd(G * W, seed=1), rnd(G * W, seed=2), rnd(E, G * W, seed=3)
    ref = torch.cat([F.silu(F.layer_norm(X[:, g * W:(g + 1) * W], (W,), gam[g * W:(g + 1) * W],
                                         bet[g * W:(g + 1) * W], 1e-5)) for g in range(G)], 1)
    (gref,) = torch.autograd.grad(ref, X, gY)
    Y = torch.empty(E, G * W, device=dev)
    call("atom_ln_silu_fwd", ptr(X.detach()), E, G * W, G, W, ptr(gam), ptr(bet), 1e-5, ptr(Y), s())
    close(Y, ref, 1e-5)
    dX = torch.empty_like(Y)
    call("atom_ln_silu_bwd", ptr(X.detach()), ptr(gY), E, G * W, G, W, ptr(gam), ptr(bet), 1e-5,
         ptr(dX), s())
    close(dX, gref, 1e-4)
    gY2 = gY.clone()
    call("atom_ln_silu_bwd", ptr(X.detach()), ptr(gY2), E, G * W, G, W, ptr(gam), ptr(bet), 1e-5,
         ptr(gY2), s())
    close(gY2, gref, 1e-4)
    N, P, C, Q = 50, 9, 64, 42
    inp, M = rnd(N, P, C), rnd(Q, P, seed=6)
    out = torch.empty(N, Q, C, device=dev)
    call("atom_node_project", ptr(inp), N, P, C, ptr(M), Q, 0, 0, ptr(out), s())
    close(out, torch.einsum("qp,npc->nqc", M, inp), 1e-5)
    back = torch.zeros(N, P, C, device=dev)
    call("atom_node_project", ptr(out), N, Q, C, ptr(M), P, 1, 1, ptr(back), s())
    close(back, torch.einsum("qp,nqc->npc", M, out), 1e-5)


def test_node_project_any_width_and_silu_bwd():
    """node_project with a P that has no compiled specialisation; silu_bwd on a multiple of 4
    (float4 path), an odd length (scalar path) and in place."""
    N, P, C, Q = 31, 7, 40, 5
    inp, M = rnd(N, P, C), rnd(Q, P, seed=6)
    out = torch.empty(N, Q, C, device=dev)
    call("atom_node_project", ptr(inp), N, P, C, ptr(M), Q, 0, 0, ptr(out), s())
    close(out, torch.einsum("qp,npc->nqc", M, inp), 1e-5)
    for n in (4096, 1001):
        g, pre = rnd(n, seed=7), rnd(n, seed=8)
        x = pre.clone().requires_grad_()
        (ref,) = torch.autograd.grad(F.silu(x), x, g)
        o = torch.empty(n, device=dev)
        call("atom_silu_bwd", ptr(g), ptr(pre), n, ptr(o), s())
        close(o, ref, 1e-5)
        call("atom_silu_bwd", ptr(g), ptr(pre), n, ptr(g), s())
        close(g, ref, 1e-5)


def test_segment_sum_deterministic():
    v = rnd(100003)
    sp = torch.tensor([0, 5, 5, 70000, 100003], dtype=torch.int32, device=dev)
    out = torch.empty(4, device=dev)
    call("atom_segment_sum", ptr(v), v.numel(), ptr(sp), 4, ptr(out), s())
    ref = torch.stack([v[0:5].sum(), v[5:5].sum(), v[5:70000].sum(), v[70000:].sum()])
    close(out, ref, 1e-5)
    out2 = torch.empty(4, device=dev)
    call("atom_segment_sum", ptr(v), v.numel(), ptr(sp), 4, ptr(out2), s())
    assert torch.equal(out, out2)


@pytest.mark.parametrize("W", [256, 1024])
def test_csr_sum_orders_and_scales(W):
    """Orb's segmented sums: out[n] (+)= sum over the CSR rows of node n (optionally through an
    edge-id list, optionally scaled per edge), as the plain sum in CSR order."""
    g = torch.Generator().manual_seed(3)
    N = 37
    deg = torch.randint(0, 10, (N,), generator=g)
    ptr_ = torch.cat([torch.zeros(1, dtype=torch.long), deg.cumsum(0)])
    E = int(ptr_[-1])
    X = rnd(E, W + 8, seed=4)
    sc = rnd(E, 2, seed=5)
    eid = torch.randperm(E, generator=g)
    ptr_d, eid_d = ptr_.to(dev, torch.int32), eid.to(dev, torch.int32)   # kept alive
    for use_eid in (False, True):
        for use_scale in (False, True):
            out = rnd(N, W, seed=6)
            base = out.clone()
            call("atom_csr_sum", ptr(X), W + 8, ptr(sc) if use_scale else None, 2,
                 ptr(ptr_d), ptr(eid_d) if use_eid else None,
                 N, W, ptr(out), W, 1, s())
            ref = base.double().clone()
            for n in range(N):
                for k in range(int(ptr_[n]), int(ptr_[n + 1])):
                    e = int(eid[k]) if use_eid else k
                    w = float(sc[e, 0]) if use_scale else 1.0
                    ref[n] += w * X[e, :W].double()
            close(out, ref, 1e-5)


@pytest.mark.parametrize("N,C", [(1, 4), (1002, 256), (37, 70)])
def test_col_mean_fixed_order(N, C):
    """out[c] = scale * sum_n X[n, c] over a padded row stride; the same result twice."""
    X = rnd(N, C + 12, seed=9)
    out = torch.empty(C, device=dev)
    call("atom_col_mean", ptr(X), C + 12, N, C, 1.0 / N, ptr(out), s())
    close(out, X[:, :C].double().sum(0) / N, 1e-6)
    out2 = torch.empty(C, device=dev)
    call("atom_col_mean", ptr(X), C + 12, N, C, 1.0 / N, ptr(out2), s())
    assert torch.equal(out, out2)
