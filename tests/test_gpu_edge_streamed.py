"""The edge kernels against plain torch fp32 references of the same ops, through the C-ABI.

At C = 128 `atom_rotate_in` and `atom_rotate_in_bwd_edge` run the persistent kernels that stream
each edge's rows through per-warp shared-memory rings (cp.async.bulk); other widths run the
warp-per-edge kernels. Both are checked here on edge counts that leave the last warps of the
persistent grid with fewer edges than the others, and on a single edge. The gate kernels run on
float4 when H is a multiple of 4 and per element otherwise; both are checked too.
"""
import ctypes

import pytest
import torch

from tt_atom import _lib as L
from tt_atom._lib import call, ptr

pytestmark = pytest.mark.gpu
dev = "cuda"

# m-primed row r: degree and offset of its nonzeros in the packed [E, 35] coefficients
ROW_DEG = [0, 1, 2, 1, 2, 1, 2, 2, 2]
ROW_OFF = [0, 1, 4, 9, 12, 17, 20, 25, 30]
RAD_SLICE = [0, 1, 2, 3, 4, 3, 4, 5, 5]    # radial slice multiplying row r
GATE_ROW = [None, 0, 1, 0, 1, 0, 1, 1, 1]


def wigner_dense(coef):
    """[E, 35] packed rows -> dense [E, 9, 9] (row r, columns of its degree block)."""
    E = coef.shape[0]
    W = torch.zeros(E, 9, 9, dtype=coef.dtype, device=coef.device)
    for r in range(9):
        l, o = ROW_DEG[r], ROW_OFF[r]
        W[:, r, l * l:l * l + 2 * l + 1] = coef[:, o:o + 2 * l + 1]
    return W


def pack(gW):
    """dense [E, 9, 9] adjoint -> packed [E, 35] (the nonzero positions only)."""
    out = torch.zeros(gW.shape[0], 35, dtype=gW.dtype, device=gW.device)
    for r in range(9):
        l, o = ROW_DEG[r], ROW_OFF[r]
        out[:, o:o + 2 * l + 1] = gW[:, r, l * l:l * l + 2 * l + 1]
    return out


def case(E, N, C, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(N, 9, C, generator=g)
    src = torch.randint(0, N, (E,), generator=g, dtype=torch.int32)
    tgt = torch.sort(torch.randint(0, N, (E,), generator=g, dtype=torch.int32)).values
    coef = torch.randn(E, 35, generator=g)
    ldr = 6 * 2 * C + 8                       # a wider radial buffer, slices from column 4
    rad = torch.randn(E, ldr, generator=g)
    return x, src, tgt, coef, rad, ldr, 4


def rotate_in_ref(x, src, tgt, coef, rad, ldr, rad_col, C):
    W = wigner_dense(coef.double())
    xs, xt = x.double()[src.long()], x.double()[tgt.long()]
    rot = torch.cat([torch.einsum("erj,ejc->erc", W, xs), torch.einsum("erj,ejc->erc", W, xt)], 2)
    sl = rad.double()[:, rad_col:rad_col + 12 * C].reshape(-1, 6, 2 * C)
    mult = sl[:, RAD_SLICE, :]
    return rot, rot * mult, mult


@pytest.mark.parametrize("E,N,C", [(1, 3, 128), (1237, 97, 128), (5003, 401, 128), (777, 60, 32)])
def test_rotate_in_matches_torch(E, N, C):
    x, src, tgt, coef, rad, ldr, rad_col = case(E, N, C, seed=E)
    _, A_ref, _ = rotate_in_ref(x, src, tgt, coef, rad, ldr, rad_col, C)
    d = [t.to(dev) for t in (x, src, tgt, coef, rad)]
    A = torch.full((E, 9 * 2 * C), float("nan"), device=dev)
    call("atom_rotate_in", ptr(d[0]), ptr(d[1]), ptr(d[2]), ptr(d[3]), E, C, ptr(d[4]), ldr,
         rad_col, None, ptr(A), L.stream_ptr())
    torch.cuda.synchronize()
    err = (A.double().cpu().reshape(E, 9, 2 * C) - A_ref).abs().max().item()
    assert err <= 1e-5 * max(A_ref.abs().max().item(), 1.0), err


@pytest.mark.parametrize("E,N,C", [(1, 3, 128), (1237, 97, 128), (5003, 401, 128), (777, 60, 32)])
def test_rotate_in_bwd_edge_matches_torch(E, N, C):
    x, src, tgt, coef, rad, ldr, rad_col = case(E, N, C, seed=E + 1)
    g = torch.Generator().manual_seed(E + 2)
    gA = torch.randn(E, 9, 2 * C, generator=g)
    g_coef0 = torch.randn(E, 35, generator=g)       # adjoints accumulated by earlier kernels
    rot, _, mult = rotate_in_ref(x, src, tgt, coef, rad, ldr, rad_col, C)
    gAd = gA.double()
    g_rot_ref = gAd * mult
    gm = gAd * rot                                   # adjoint of the multiplier per row
    g_rad_ref = torch.zeros(E, 6, 2 * C, dtype=torch.float64)
    for r in range(9):
        g_rad_ref[:, RAD_SLICE[r]] += gm[:, r]
    xs, xt = x.double()[src.long()], x.double()[tgt.long()]
    gW = (torch.einsum("erc,ejc->erj", g_rot_ref[:, :, :C], xs)
          + torch.einsum("erc,ejc->erj", g_rot_ref[:, :, C:], xt))
    g_coef_ref = g_coef0.double() + pack(gW)
    d = [t.to(dev) for t in (x, src, tgt, coef, rad, gA)]
    g_rot = torch.full((E, 9 * 2 * C), float("nan"), device=dev)
    g_rad = torch.full((E, ldr), float("nan"), device=dev)
    g_coef = g_coef0.clone().to(dev)
    call("atom_rotate_in_bwd_edge", ptr(d[5]), None, ptr(d[4]), ldr, rad_col, ptr(d[0]),
         ptr(d[1]), ptr(d[2]), ptr(d[3]), E, C, ptr(g_rot), ptr(g_rad), ptr(g_coef),
         L.stream_ptr())
    torch.cuda.synchronize()
    code = ctypes.c_int(-1)
    call("atom_device_error", ctypes.byref(code), L.stream_ptr())
    assert code.value == 0

    def chk(got, ref):
        err = (got.double().cpu() - ref).abs().max().item()
        assert err <= 1e-5 * max(ref.abs().max().item(), 1.0), err

    chk(g_rot.reshape(E, 9, 2 * C), g_rot_ref)
    chk(g_rad[:, rad_col:rad_col + 12 * C].reshape(E, 6, 2 * C), g_rad_ref)
    chk(g_coef, g_coef_ref)


@pytest.mark.parametrize("E,H", [(3001, 128), (513, 36), (257, 30)])
def test_gate_fwd_bwd_match_torch(E, H):
    g = torch.Generator().manual_seed(H)
    Y = torch.randn(E, 11 * H, generator=g)
    gG = torch.randn(E, 9 * H, generator=g)
    y = Y.double().reshape(E, 11, H)
    s = torch.sigmoid(y[:, :2])
    G_ref = torch.empty(E, 9, H, dtype=torch.float64)
    G_ref[:, 0] = torch.nn.functional.silu(y[:, 2])
    for r in range(1, 9):
        G_ref[:, r] = y[:, 2 + r] * s[:, GATE_ROW[r]]
    yr = y.clone().requires_grad_(True)
    sr = torch.sigmoid(yr[:, :2])
    Gr = torch.stack([torch.nn.functional.silu(yr[:, 2])]
                     + [yr[:, 2 + r] * sr[:, GATE_ROW[r]] for r in range(1, 9)], 1)
    (gY_ref,) = torch.autograd.grad(Gr, yr, gG.double().reshape(E, 9, H))
    Yd, gGd = Y.to(dev), gG.to(dev)
    G = torch.full((E, 9 * H), float("nan"), device=dev)
    gY = torch.full((E, 11 * H), float("nan"), device=dev)
    call("atom_gate_fwd", ptr(Yd), E, H, ptr(G), L.stream_ptr())
    call("atom_gate_bwd", ptr(Yd), ptr(gGd), E, H, ptr(gY), L.stream_ptr())
    torch.cuda.synchronize()
    for got, ref in ((G.reshape(E, 9, H), G_ref), (gY.reshape(E, 11, H), gY_ref)):
        err = (got.double().cpu() - ref).abs().max().item()
        assert err <= 1e-5 * max(ref.abs().max().item(), 1.0), err
