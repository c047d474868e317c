"""The eSCN-MD energy + force + stress engine on the GPU.

``UMAEngine`` owns the device copies of the (re-laid-out) weights; ``Workspace`` owns every
activation buffer for one graph topology. ``UMAEngine.run`` issues the whole step -- geometry,
radial MLPs, the L edgewise/atomwise blocks, the energy head, then the hand-written reverse pass
down to forces and the virial -- as a fixed sequence of C-ABI kernel launches on one stream, so
the step can be captured once in a CUDA graph and replayed (``CapturedStep``).

Reference structure followed (reference tt-atom):
  forward   tt_atom/model.py:138-247 (_Block, Backbone), tt_atom/edgewise.py:39-87,
            tt_atom/geometry.py:226-280 (geometry + edge-degree init)
  backward  tt_atom/forces.py:73-495 (rmsnorm_bw .. backbone_bw) and the host autograd finish of
            tt_atom/forces.py:545-589, here done on the GPU (geometry VJP, force/virial reduce).

Weight re-layouts done once at load time:
  * radial MLPs of all layers and of the edge-degree embedding are batched: their first linear
    is split into the Gaussian columns (one GEMM over all groups) and the source/target
    embedding columns, which are folded with the bias into per-species tables gathered in the
    GEMM epilogue;
  * each SO(2) m > 0 linear becomes one GEMM on [real | imag] with the block weight
    [[P, Q], [-Q, P]] (W^T = [P | Q]), equal to the reference's (a - d, c + b) combination;
  * transposed copies for the reverse pass.
"""
from __future__ import annotations

import dataclasses
import math

import numpy as np

import torch

from . import _lib as L
from ._lib import ptr

# kernels launched per entry point (all others launch one)
call = L.call

# "fp32": FMA-pipe GEMMs; "3xtf32": tcgen05 tensor cores with the tf32 hi/lo operand split
# (fp32-level accuracy); "3xf16": the same three products on fp16 hi/lo pairs with
# power-of-two row and column scales (fp32-level accuracy at twice the tf32 MMA rate);
# "tf32": tensor cores, one pass (looser, ~1e-3 relative per product).
PRECISIONS = {"fp32": 0, "tf32": 1, "3xtf32": 2, "3xf16": 3}


def to_host(*ts):
    """float64 host copies of several device result tensors through one device-to-host copy
    (one synchronisation instead of one per tensor); None entries stay None."""
    live = [t for t in ts if t is not None]
    if not live:
        return [None] * len(ts)
    dev = next((t.device for t in live if t.is_cuda), None)
    flag = None
    if dev is not None:
        # a GEMM whose bounded wait expired leaves its outputs incomplete: its error code is
        # read back with the results (and cleared) and the results are refused
        flag = _error_slot(dev)
        L.call("atom_device_error_take", flag.data_ptr(), L.stream_ptr())
    parts = [t.reshape(-1).to(torch.float64) for t in live]
    if flag is not None:
        parts.append(flag.to(device=parts[0].device, dtype=torch.float64))
    flat = torch.cat(parts).cpu()
    if flag is not None:
        code = int(flat[-1])
        if code != 0:
            raise RuntimeError(
                f"a bounded device-side wait in the tensor-core GEMM expired (code {code}); "
                "the results of this evaluation are incomplete and were discarded")
    out, o = [], 0
    for t in ts:
        if t is None:
            out.append(None)
            continue
        out.append(flat[o:o + t.numel()].reshape(t.shape))
        o += t.numel()
    return out


_ERROR_SLOTS = {}


def _error_slot(dev):
    """A one-int device buffer per device for the error code read back with results."""
    t = _ERROR_SLOTS.get(str(dev))
    if t is None:
        t = _ERROR_SLOTS[str(dev)] = torch.zeros(1, dtype=torch.int32, device=dev)
    return t


def upload_positions(ws, pos):
    """Copy positions into ``ws.pos``: a device tensor directly; host values through a pinned
    staging buffer of the workspace (asynchronous host-to-device copy, ordered on the current
    stream; the staging buffer is reused only after its previous copy has completed)."""
    if torch.is_tensor(pos) and pos.is_cuda:
        ws.pos.copy_(pos)
        return
    pin = getattr(ws, "_pos_pinned", None)
    if pin is None:
        ws._pos_pinned = pin = torch.empty(ws.pos.shape, dtype=torch.float32, pin_memory=True)
        ws._pos_event = torch.cuda.Event()
    else:
        ws._pos_event.synchronize()
    pin.copy_(torch.as_tensor(pos, dtype=torch.float32).reshape(pin.shape))
    ws.pos.copy_(pin, non_blocking=True)
    ws._pos_event.record()


def launch_count():
    """Kernels the library has launched so far (its own counter)."""
    n = L.ctypes.c_int64(0)
    L.call("atom_launch_count", L.ctypes.byref(n))
    return n.value


def _split_tf32(t):
    """(hi, lo): hi = t with the low 13 mantissa bits cleared, lo = t - hi (exact)."""
    hi = (t.contiguous().view(torch.int32) & -8192).view(torch.float32)
    return hi.contiguous(), (t - hi).contiguous()


def _split_f16(t):
    """Mode-3 weight halves of a K-major weight t [N, K]: per row n the power-of-two scale
    s = 2^(14 - floor(log2 max |t[n]|)) (1 for a zero row), hi = fp16(t s),
    lo = fp16((t s - hi) 2^11); returns (hi, lo, 1 / s)."""
    mx = t.abs().amax(dim=1)
    e = torch.floor(torch.log2(torch.where(mx > 0, mx, torch.ones_like(mx))))
    sh = torch.clamp(14.0 - e, -126.0, 126.0)
    s = torch.where(mx > 0, torch.exp2(sh), torch.ones_like(mx))
    y = t * s[:, None]
    hi = y.half()
    lo = ((y - hi.float()) * 2048.0).half()
    return hi.contiguous(), lo.contiguous(), (1.0 / s).contiguous()


def _dev(t, device):
    return t.detach().to(device=device, dtype=torch.float32).contiguous()


class _Groups:
    """A grouped-GEMM description (up to 8 groups) kept alive with its tensors."""

    def __init__(self, groups):
        self.keep = []
        self._tf32 = []
        self._f16 = False
        g = L.GemmGroups()
        g.ngroups = len(groups)
        for i, d in enumerate(groups):
            g.a_col[i] = d["a_col"]
            g.K[i] = d["K"]
            g.c_col[i] = d["c_col"]
            g.N[i] = d["N"]
            B = d["B"]
            g.ldb[i] = B.shape[1]
            g.t_col[i] = d.get("t_col", 0)
            g.B[i] = B.data_ptr()
            self.keep.append(B)
            # K-major copies for the tensor-core kernel (hi part, lo part)
            hi, lo = _split_tf32(B[:d["K"], :d["N"]].t().contiguous())
            g.Bt[i] = hi.data_ptr()
            g.Bt_lo[i] = lo.data_ptr()
            self.keep += [hi, lo]
            self._tf32.append((hi, lo))
            b = d.get("bias")
            g.bias[i] = b.data_ptr() if b is not None else None
            if b is not None:
                self.keep.append(b)
        self.struct = g

    def ensure_f16(self):
        """Add the fp16-pair mode's weight halves and column scales (made on first use from the
        tf32 pair, whose sum is the weight exactly); without them that mode runs as 3xTF32."""
        if not self._f16:
            for i, (hi, lo) in enumerate(self._tf32):
                h16, l16, inv = _split_f16(hi + lo)
                self.struct.Bh[i] = h16.data_ptr()
                self.struct.Bh_lo[i] = l16.data_ptr()
                self.struct.Bh_inv[i] = inv.data_ptr()
                self.keep += [h16, l16, inv]
            self._f16 = True
        return self


def _so2_blocks(W_m0, b_m0, W_m, cin, hout, extra):
    """Forward/backward grouped-GEMM weights of one SO(2) convolution (lmax = mmax = 2).

    A layout per edge: m-primed rows x cin -> columns [rows 0..2 | rows 3,4 | rows 5,6 | 7 | 8].
    Output: [extra | rows 0..8 x hout]."""
    fwd, bwd = [], []
    k0 = 3 * cin
    n0 = extra + 3 * hout
    fwd.append(dict(a_col=0, K=k0, c_col=0, N=n0, B=W_m0.t().contiguous(), bias=b_m0))
    bwd.append(dict(a_col=0, K=n0, c_col=0, N=k0, B=W_m0.contiguous()))
    a_col, c_col = k0, n0
    for m, W in enumerate(W_m, start=1):
        nc = 3 - m
        k = nc * cin            # per real/imag half
        h = nc * hout
        Wt = W.t()              # [k, 2h]
        P, Q = Wt[:, :h], Wt[:, h:]
        B = torch.cat([torch.cat([P, Q], 1), torch.cat([-Q, P], 1)], 0).contiguous()  # [2k, 2h]
        fwd.append(dict(a_col=a_col, K=2 * k, c_col=c_col, N=2 * h, B=B))
        bwd.append(dict(a_col=c_col, K=2 * h, c_col=a_col, N=2 * k, B=B.t().contiguous()))
        a_col += 2 * k
        c_col += 2 * h
    return fwd, bwd


class UMAEngine:
    """Device-resident eSCN-MD (UMA, lmax = mmax = 2, grid feed-forward) for E, F and stress."""

    def __init__(self, weights, cfg, tables, device="cuda", precision="fp32"):
        if cfg.get("lmax", 2) != 2 or cfg.get("mmax", 2) != 2:
            raise RuntimeError("this build implements lmax = mmax = 2 (uma-s shape) only")
        self.ff = cfg.get("ff_type", "grid")
        if self.ff not in ("grid", "spectral"):
            raise RuntimeError(f"feed-forward type {self.ff!r} is not implemented")
        L.lib()
        self.device = torch.device(device)
        self.cfg = dict(cfg)
        self.precision = PRECISIONS[precision]
        C, H = cfg["sphere_channels"], cfg["hidden_channels"]
        EC, NB, NL = cfg["edge_channels"], cfg["num_distance_basis"], cfg["num_layers"]
        self.C, self.H, self.EC, self.NB, self.NL = C, H, EC, NB, NL
        self.cutoff = float(cfg["cutoff"])
        w = {k: v.float() for k, v in weights.items()}
        dev = self.device
        d = lambda t: _dev(t, dev)  # noqa: E731

        # fixed tables
        self.jd1 = L.host_f32(w["Jd_1"].reshape(-1).tolist())
        self.jd2 = L.host_f32(w["Jd_2"].reshape(-1).tolist())
        to_m = tables["to_m"]
        self.perm9 = L.host_i32(to_m.abs().argmax(dim=1).tolist())
        self.offset = d(tables["gauss_offset"].reshape(-1))
        self.coeff = float(tables["gauss_coeff"].reshape(-1)[0])
        tg = tables["to_grid_mat"].reshape(-1, 9)
        fg = tables["from_grid_mat"].reshape(-1, 9)
        self.npts = tg.shape[0]
        self.TG, self.FG = d(tg), d(fg)

        # ---- radial MLPs: groups = layers' so2_conv_1 radial functions + edge-degree
        prefixes = [f"blocks.{i}.edge_wise.so2_conv_1.rad_func" for i in range(NL)]
        prefixes.append("edge_degree_embedding.rad_func")
        G = len(prefixes)
        if G > 8:
            raise RuntimeError("at most 7 layers are supported by the batched radial GEMM")
        self.G = G
        src_emb, tgt_emb = w["source_embedding.weight"], w["target_embedding.weight"]
        w0g, ts, tt, ln1g, ln1b, ln2g, ln2b = [], [], [], [], [], [], []
        f2, f2b, f3, f3b, r_out = [], [], [], [], []
        for p in prefixes:
            W0, b0 = w[f"{p}.net.0.weight"], w[f"{p}.net.0.bias"]      # [EC, NB + 2 EC]
            w0g.append(W0[:, :NB])
            ts.append(src_emb @ W0[:, NB:NB + EC].t() + b0)
            tt.append(tgt_emb @ W0[:, NB + EC:].t())
            ln1g.append(w[f"{p}.net.1.weight"]); ln1b.append(w[f"{p}.net.1.bias"])
            ln2g.append(w[f"{p}.net.4.weight"]); ln2b.append(w[f"{p}.net.4.bias"])
            f2.append(w[f"{p}.net.3.weight"]); f2b.append(w[f"{p}.net.3.bias"])
            f3.append(w[f"{p}.net.6.weight"]); f3b.append(w[f"{p}.net.6.bias"])
            r_out.append(w[f"{p}.net.6.weight"].shape[0])
        self.W0g_cat = d(torch.cat(w0g, 0))                       # [G*EC, NB]
        self.rad1 = _Groups([dict(a_col=0, K=NB, c_col=0, N=G * EC,
                                  B=d(torch.cat(w0g, 0).t()))])
        self.Tsrc, self.Ttgt = d(torch.cat(ts, 1)), d(torch.cat(tt, 1))   # [nel, G*EC]
        self.ln1g, self.ln1b = d(torch.cat(ln1g)), d(torch.cat(ln1b))
        self.ln2g, self.ln2b = d(torch.cat(ln2g)), d(torch.cat(ln2b))
        self.rad2 = _Groups([dict(a_col=g * EC, K=EC, c_col=g * EC, N=EC, B=d(f2[g].t()),
                                  bias=d(f2b[g])) for g in range(G)])
        self.rad2_bw = _Groups([dict(a_col=g * EC, K=EC, c_col=g * EC, N=EC, B=d(f2[g]))
                                for g in range(G)])
        self.rad_off = [0]
        for o in r_out:
            self.rad_off.append(self.rad_off[-1] + o)
        self.ldr = self.rad_off[-1]
        self.rad3 = _Groups([dict(a_col=g * EC, K=EC, c_col=self.rad_off[g], N=r_out[g],
                                  B=d(f3[g].t()), bias=d(f3b[g])) for g in range(G)])
        self.rad3_bw = _Groups([dict(a_col=self.rad_off[g], K=r_out[g], c_col=g * EC, N=EC,
                                     B=d(f3[g])) for g in range(G)])
        self.rad1_bw = _Groups([dict(a_col=0, K=G * EC, c_col=0, N=NB, B=self.W0g_cat)])
        # one group at a time, for receiver-chunked execution (a layer's radial function is
        # recomputed per chunk instead of storing [E, 6528] radial outputs and their adjoint)
        self.radg = []
        for g in range(G):
            self.radg.append(dict(
                r1=_Groups([dict(a_col=0, K=NB, c_col=0, N=EC, B=d(w0g[g].t()), t_col=g * EC)]),
                r2=_Groups([dict(a_col=0, K=EC, c_col=0, N=EC, B=d(f2[g].t()), bias=d(f2b[g]))]),
                r3=_Groups([dict(a_col=0, K=EC, c_col=0, N=r_out[g], B=d(f3[g].t()),
                                 bias=d(f3b[g]))]),
                r3_bw=_Groups([dict(a_col=0, K=r_out[g], c_col=0, N=EC, B=d(f3[g]))]),
                r2_bw=_Groups([dict(a_col=0, K=EC, c_col=0, N=EC, B=d(f2[g]))]),
                r1_bw=_Groups([dict(a_col=0, K=EC, c_col=0, N=NB, B=d(w0g[g]))]),
                width=r_out[g]))
        for i in range(NL):
            assert r_out[i] == 12 * C, "so2_conv_1 radial output must be 6 * 2C"
        assert r_out[NL] == 3 * C, "edge-degree radial output must be 3C"

        # ---- per block
        self.blocks = []
        for i in range(NL):
            p = f"blocks.{i}"
            e1 = f"{p}.edge_wise.so2_conv_1"
            e2 = f"{p}.edge_wise.so2_conv_2"
            f1, b1 = _so2_blocks(d(w[f"{e1}.fc_m0.weight"]), d(w[f"{e1}.fc_m0.bias"]),
                                 [d(w[f"{e1}.so2_m_conv.{m}.fc.weight"]) for m in range(2)],
                                 2 * C, H, 2 * H)
            f2_, b2_ = _so2_blocks(d(w[f"{e2}.fc_m0.weight"]), d(w[f"{e2}.fc_m0.bias"]),
                                   [d(w[f"{e2}.so2_m_conv.{m}.fc.weight"]) for m in range(2)],
                                   H, C, 0)
            blk = dict(
                n1w=d(w[f"{p}.norm_1.affine_weight"]), n1b=d(w[f"{p}.norm_1.affine_bias"]),
                n2w=d(w[f"{p}.norm_2.affine_weight"]), n2b=d(w[f"{p}.norm_2.affine_bias"]),
                so2_1=_Groups(f1), so2_1_bw=_Groups(b1), so2_2=_Groups(f2_), so2_2_bw=_Groups(b2_),
                # the same so2_2 weights addressing the so2_1 output's rows directly (the gate
                # applied inside the GEMM: atom_gemm_gated)
                so2_2g=_Groups([dict(gr, a_col=gr["a_col"] + 2 * H) for gr in f2_]))
            a = f"{p}.atom_wise"
            if self.ff == "grid":
                for key, gi in (("ga", 0), ("gb", 2), ("gc", 4)):
                    W = w[f"{a}.grid_mlp.{gi}.weight"]
                    blk[key] = _Groups([dict(a_col=0, K=C, c_col=0, N=C, B=d(W.t()))])
                    blk[key + "_bw"] = _Groups([dict(a_col=0, K=C, c_col=0, N=C, B=d(W))])
            else:
                blk.update(self._spectral_weights(w, a, d))
            self.blocks.append(blk)
        self.nfw, self.nfb = d(w["norm.affine_weight"]), d(w["norm.affine_bias"])
        E0, E2, E4 = w["energy_block.0.weight"], w["energy_block.2.weight"], w["energy_block.4.weight"]
        self.eh0 = _Groups([dict(a_col=0, K=C, c_col=0, N=H, B=d(E0.t()),
                                 bias=d(w["energy_block.0.bias"]))])
        self.eh2 = _Groups([dict(a_col=0, K=H, c_col=0, N=H, B=d(E2.t()),
                                 bias=d(w["energy_block.2.bias"]))])
        self.eh4 = _Groups([dict(a_col=0, K=H, c_col=0, N=1, B=d(E4.t()),
                                 bias=d(w["energy_block.4.bias"]))])
        self.eh2_bw = _Groups([dict(a_col=0, K=H, c_col=0, N=H, B=d(E2))])
        self.eh0_bw = _Groups([dict(a_col=0, K=H, c_col=0, N=C, B=d(E0))])
        self.eh4_row = d(E4.reshape(-1))
        self.sphere = d(w["sphere_embedding.weight"])
        self._w_host = w

    def _spectral_weights(self, w, a, d):
        """Grouped-GEMM weights of one spectral feed-forward (tt_atom/spectral.py:41-188): the
        scalar MLP on l = 0 and the two SO3 linears as one group per coefficient (weight of the
        coefficient's degree, bias on coefficient 0), split into launches of at most 8 groups."""
        C, H = self.C, self.H
        lc = [0, 1, 1, 1, 2, 2, 2, 2, 2]
        Ws, bs = w[f"{a}.scalar_mlp.0.weight"], w[f"{a}.scalar_mlp.0.bias"]
        W1, b1 = w[f"{a}.so3_linear_1.weight"], w[f"{a}.so3_linear_1.bias"]
        W2, b2 = w[f"{a}.so3_linear_2.weight"], w[f"{a}.so3_linear_2.bias"]
        bias1, bias2 = d(b1), d(b2)

        def split(gs):
            return [_Groups(gs[:5]), _Groups(gs[5:])]
        return dict(
            sm=_Groups([dict(a_col=0, K=C, c_col=0, N=Ws.shape[0], B=d(Ws.t()), bias=d(bs))]),
            sm_bw=_Groups([dict(a_col=0, K=Ws.shape[0], c_col=0, N=C, B=d(Ws))]),
            so3_1=split([dict(a_col=c * C, K=C, c_col=c * H, N=H, B=d(W1[lc[c]].t()),
                              bias=bias1 if c == 0 else None) for c in range(9)]),
            so3_1_bw=split([dict(a_col=c * H, K=H, c_col=c * C, N=C, B=d(W1[lc[c]]))
                            for c in range(9)]),
            so3_2=split([dict(a_col=c * H, K=H, c_col=c * C, N=C, B=d(W2[lc[c]].t()),
                              bias=bias2 if c == 0 else None) for c in range(9)]),
            so3_2_bw=split([dict(a_col=c * C, K=C, c_col=c * H, N=H, B=d(W2[lc[c]]))
                            for c in range(9)]))

    # ------------------------------------------------------------------------------ helpers
    _scratch = None

    def _gemm(self, A, lda, M, groups, Cout, ldc, *, Cpre=None, T1=None, T2=None, idx1=None,
              idx2=None, ldt=0, act=0, accumulate=0, stream=0):
        # the workspace's scratch lets node-level launches (few rows) split K over more CTAs
        sc = self._scratch
        prec = self.precision
        if prec == 3:
            groups.ensure_f16()
        call("atom_gemm_ex", ptr(A), lda, M, groups.struct, ptr(Cout), ldc, ptr(Cpre), ptr(T1),
             ptr(T2), ptr(idx1), ptr(idx2), ldt, act, accumulate, prec, ptr(sc),
             sc.numel() if sc is not None else 0, stream)

    # True: the gate of the edgewise block applied inside the so2_2 GEMM (tensor-core
    # precisions, atom_gemm_gated); False (default): the standalone gate kernel, then the GEMM.
    # Same results bit for bit. Measured on the 2,000-atom step: 17.53 ms fused against
    # 17.18 ms separate (3xTF32), 18.58 against 18.16 ms (fp16 pair): the gating tile each K
    # stage then reads adds a quarter to the GEMM's per-stage operand traffic, which costs more
    # than the standalone pass over HBM.
    fuse_gate = False

    def _gate_so2_2(self, ws, Y1, E, b, out, s):
        """so2_2 on the gated so2_1 output Y1 [E, 11H] into ``out`` [E, 9C]."""
        H, C = self.H, self.C
        if self.fuse_gate and self.precision >= 2 and H % 32 == 0:
            sc = self._scratch
            if self.precision == 3:
                b["so2_2g"].ensure_f16()
            rc = L.lib().atom_gemm_gated(ptr(Y1), 11 * H, E, b["so2_2g"].struct, H, ptr(out),
                                         9 * C, self.precision, ptr(sc),
                                         sc.numel() if sc is not None else 0, s)
            if rc == 0:
                return
            if rc != L.ATOM_ERR_UNSUPPORTED:
                raise L.AtomError("atom_gemm_gated", rc)
        call("atom_gate_fwd", ptr(Y1), E, H, ptr(ws.Gt), s)
        self._gemm(ws.Gt, 9 * H, E, b["so2_2"], out, 9 * C, stream=s)

    def workspace_bytes(self, N, E, chunk_edges=None):
        """Approximate device bytes of a workspace for N atoms and E edges (unchunked, or
        with receiver chunks of ``chunk_edges`` edges)."""
        C, H, EC, NB, G, NL, P = self.C, self.H, self.EC, self.NB, self.G, self.NL, self.npts
        node = N * (9 * C * (3 * NL + 9) + (2 * NL + 3) * P * C + 8 * H + 2 * C)
        geo = E * 2 * (NB + 39)
        if chunk_edges is None:
            edge = E * (4 * G * EC + 2 * self.ldr + NL * (11 * H + 9 * C) + 45 * C + 20 * H)
        else:
            RW = max(r["width"] for r in self.radg)
            edge = min(chunk_edges, E) * (4 * EC + 2 * RW + 31 * H + 54 * C)
        return 4 * (node + geo + edge)

    def choose_chunk_edges(self, graph, budget_bytes=None):
        """None when the unchunked workspace fits ``budget_bytes`` (default: 85 % of the
        device's free memory), else the largest receiver-chunk size that does."""
        N, E = graph.N, graph.E
        if budget_bytes is None:
            budget_bytes = 0.85 * torch.cuda.mem_get_info(self.device)[0]
        if self.workspace_bytes(N, E) <= budget_bytes:
            return None
        fixed = self.workspace_bytes(N, E, chunk_edges=0)
        per_edge = self.workspace_bytes(N, E, chunk_edges=1) - fixed
        max_in = int((graph.recv_ptr[1:] - graph.recv_ptr[:-1]).max()) if N else 1
        k = int((budget_bytes - fixed) // per_edge)
        if k < max(max_in, 1):
            raise MemoryError(f"{N} atoms / {E} edges do not fit in {budget_bytes / 1e9:.1f} GB "
                              f"even in receiver chunks (fixed part {fixed / 1e9:.1f} GB)")
        return min(k, E)

    def workspace(self, graph, sys_emb, chunk_edges=None):
        """Device buffers for one topology. With ``chunk_edges`` the edge stages run over
        contiguous receiver chunks of at most that many edges (recomputed in the reverse
        pass), so per-edge storage is the geometry only; see ``Workspace``."""
        return Workspace(self, graph, sys_emb, chunk_edges=chunk_edges)

    def launches_per_step(self, ws, forces=True, virial=True):
        """Number of this library's kernels one ``run`` launches (counted, not estimated)."""
        torch.cuda.synchronize()
        c0 = launch_count()
        self.run(ws, ws.pos, forces=forces, virial=virial)
        torch.cuda.synchronize()
        return launch_count() - c0

    def so2_flop(self, E):
        """Algorithmic FLOPs of one forward so2_1 grouped GEMM over E edges."""
        C, H = self.C, self.H
        mac = 6 * C * 5 * H + 8 * C * 4 * H + 4 * C * 2 * H
        return 2.0 * E * mac

    def time_kernels(self, ws, reps=5):
        """Average device time of the dominant kernel (the layer-0 so2_1 grouped GEMM), timed
        with CUDA events on the stream it is launched on."""
        st = torch.cuda.Stream(device=self.device)
        st.wait_stream(torch.cuda.current_stream())
        s = st.cuda_stream
        E = ws.graph.E
        b = self.blocks[0]
        with torch.cuda.stream(st):
            self._gemm(ws.A1, 18 * self.C, E, b["so2_1"], ws.Y1[0], 11 * self.H, stream=s)
            t0 = torch.cuda.Event(enable_timing=True)
            t1 = torch.cuda.Event(enable_timing=True)
            t0.record(st)
            for _ in range(reps):
                self._gemm(ws.A1, 18 * self.C, E, b["so2_1"], ws.Y1[0], 11 * self.H, stream=s)
            t1.record(st)
        st.synchronize()
        torch.cuda.current_stream().wait_stream(st)
        return dict(name="so2_conv_1 grouped GEMM", ms=t0.elapsed_time(t1) / reps,
                    flop=self.so2_flop(E))

    def time_edge_kernel(self, ws, reps=5):
        """Average device time of the layer-0 rotate-in edge kernel (Wigner rotation of both
        node rows times the radial slices, HBM-bound) with its algorithmic bytes per launch:
        node rows read once, radial slices, coefficients and indices read, A written."""
        st = torch.cuda.Stream(device=self.device)
        st.wait_stream(torch.cuda.current_stream())
        s = st.cuda_stream
        g = ws.graph
        E, N, C = g.E, g.N, self.C

        def launch():
            call("atom_rotate_in", ptr(ws.nb[0]), ptr(g.src), ptr(g.tgt), ptr(ws.coef), E, C,
                 ptr(ws.RAD), self.ldr, self.rad_off[0], None, ptr(ws.A1), s)
        with torch.cuda.stream(st):
            launch()
            t0 = torch.cuda.Event(enable_timing=True)
            t1 = torch.cuda.Event(enable_timing=True)
            t0.record(st)
            for _ in range(reps):
                launch()
            t1.record(st)
        st.synchronize()
        torch.cuda.current_stream().wait_stream(st)
        nbytes = 4 * (N * 9 * C + E * (6 * 2 * C + 35 + 2 + 9 * 2 * C))
        return dict(name="rotate_in (Wigner rotation x radial)", ms=t0.elapsed_time(t1) / reps,
                    bytes=nbytes)

    def time_edge_kernels(self, ws, reps=5, layer=0):
        """CUDA-event time per launch of each HBM-bound edge kernel of one layer (forward and
        reverse), run on ``ws``'s current buffers, with its algorithmic bytes per launch (each
        input and output array once; node rows once per table) and the achieved rate. Needs a
        workspace that has run a full step (unchunked)."""
        g = ws.graph
        E, N, C, H, i = g.E, g.N, self.C, self.H, layer
        st = torch.cuda.Stream(device=self.device)
        st.wait_stream(torch.cuda.current_stream())
        s = st.cuda_stream
        nodes = N * 9 * C
        kern = [
            ("rotate_in", lambda: call(
                "atom_rotate_in", ptr(ws.nb[i]), ptr(g.src), ptr(g.tgt), ptr(ws.coef), E, C,
                ptr(ws.RAD), self.ldr, self.rad_off[i], None, ptr(ws.A1), s),
             nodes + E * (12 * C + 35 + 2 + 18 * C)),
            ("gate_fwd", lambda: call("atom_gate_fwd", ptr(ws.Y1[i]), E, H, ptr(ws.Gt), s),
             E * 20 * H),
            ("rotate_back_reduce", lambda: call(
                "atom_rotate_back_reduce", ptr(ws.Y2[i]), ptr(ws.coef), ptr(ws.env), N, C,
                ptr(g.recv_ptr), ptr(ws.x[i]), ptr(ws.xm[i]), s),
             E * (9 * C + 35 + 1) + 2 * nodes + N),
            ("rotate_back_bwd", lambda: call(
                "atom_rotate_back_bwd", ptr(ws.gx), ptr(g.tgt), ptr(ws.coef), ptr(ws.env),
                ptr(ws.Y2[i]), E, C, ptr(ws.gY2), ptr(ws.g_env), ptr(ws.g_coef), s),
             nodes + E * (9 * C + 2 * 35 + 2 + 1 + 9 * C)),
            ("gate_bwd", lambda: call("atom_gate_bwd", ptr(ws.Y1[i]), ptr(ws.Gt), E, H,
                                      ptr(ws.gY1), s), E * 31 * H),
            ("rotate_in_bwd_edge", lambda: call(
                "atom_rotate_in_bwd_edge", ptr(ws.A1), None, ptr(ws.RAD), self.ldr,
                self.rad_off[i], ptr(ws.nb[i]), ptr(g.src), ptr(g.tgt), ptr(ws.coef), E, C,
                ptr(ws.grot), ptr(ws.gRAD), ptr(ws.g_coef), s),
             nodes + E * (18 * C + 12 * C + 2 * 35 + 2 + 18 * C + 12 * C)),
            ("rotate_in_bwd_node", lambda: call(
                "atom_rotate_in_bwd_node", ptr(ws.grot), ptr(ws.coef), N, C, ptr(g.recv_ptr),
                ptr(g.send_ptr), ptr(g.send_eid), 0, ptr(ws.gn), s),
             E * (18 * C + 2 * 35 + 1) + 2 * N + nodes),
        ]
        out = []
        with torch.cuda.stream(st):
            for name, fn, floats in kern:
                fn()
                t0 = torch.cuda.Event(enable_timing=True)
                t1 = torch.cuda.Event(enable_timing=True)
                t0.record(st)
                for _ in range(reps):
                    fn()
                t1.record(st)
                st.synchronize()
                ms = t0.elapsed_time(t1) / reps
                out.append(dict(kernel=name, ms=ms, bytes=4 * floats,
                                gbs=4 * floats / (ms / 1e3) / 1e9))
        torch.cuda.current_stream().wait_stream(st)
        return out

    # --------------------------------------------------------------------------------- step
    def run(self, ws, pos, forces=True, virial=False, stream=None):
        """One E (+F, +virial) evaluation for ``pos`` [N, 3] (device fp32) on ``ws``'s graph.
        Results land in ``ws.energy`` [nsys], ``ws.forces`` [N, 3], ``ws.virial`` [3, 3]."""
        for _ in self.steps(ws, pos, forces, virial, stream):
            pass

    def steps(self, ws, pos, forces=True, virial=False, stream=None):
        """``run`` as a generator that pauses where a spatially partitioned caller must
        exchange halo rows: ("x", i) after layer i's input features x[i] are computed (halo
        rows must then be overwritten by their owners' values), ("gx", i) after the adjoint of
        x[i] is complete (halo rows must be sent to and added by their owners, then zeroed),
        and ("forces", None) after the forces (halo rows' partial forces belong to owners)."""
        s = L.stream_ptr(stream)
        g = ws.graph
        N, E = g.N, g.E
        C, H, EC, NB, G = self.C, self.H, self.EC, self.NB, self.G
        self._scratch = ws.gemm_scratch
        if pos.data_ptr() != ws.pos.data_ptr():
            ws.pos.copy_(pos)
        # ---------------- geometry
        call("atom_edge_geometry", ptr(ws.pos), ptr(g.src), ptr(g.tgt), ptr(g.img),
             ptr(g.shifts), E, self.jd1, self.jd2, self.perm9, ptr(self.offset), NB, self.coeff,
             self.cutoff, ptr(ws.coef), ptr(ws.gauss), ptr(ws.env), ptr(ws.ev), None, s)
        if ws.chunks is None:
            # ---------------- radial MLPs (all groups at once)
            self._gemm(ws.gauss, NB, E, self.rad1, ws.R0, G * EC, T1=self.Tsrc, T2=self.Ttgt,
                       idx1=g.zs, idx2=g.zt, ldt=G * EC, stream=s)
            call("atom_ln_silu_fwd", ptr(ws.R0), E, G * EC, G, EC, ptr(self.ln1g),
                 ptr(self.ln1b), 1e-5, ptr(ws.H1), s)
            self._gemm(ws.H1, G * EC, E, self.rad2, ws.R1, G * EC, stream=s)
            call("atom_ln_silu_fwd", ptr(ws.R1), E, G * EC, G, EC, ptr(self.ln2g),
                 ptr(self.ln2b), 1e-5, ptr(ws.H2), s)
            self._gemm(ws.H2, G * EC, E, self.rad3, ws.RAD, self.ldr, stream=s)
            # ---------------- edge-degree node init
            ede = ws.RAD[:, self.rad_off[self.NL]:]
            call("atom_edge_degree_fwd", ptr(ede), self.ldr, ptr(ws.coef), ptr(ws.env),
                 ptr(ws.l0), N, C, ptr(g.recv_ptr), 5.0, ptr(ws.x[0]), s)
        else:
            for ch in ws.chunks:
                self._radial_group_fwd(ws, self.NL, ch, s)
                call("atom_edge_degree_fwd", ptr(ws.RAD), ws.RAD.shape[1],
                     ptr(ws.coef[ch.e0:]), ptr(ws.env[ch.e0:]), ptr(ws.l0[ch.n0:]),
                     ch.n1 - ch.n0, C, ptr(ch.rp_local), 5.0, ptr(ws.x[0][ch.n0:]), s)
        yield ("x", 0)
        # ---------------- blocks
        for i, b in enumerate(self.blocks):
            x, nb = ws.x[i], ws.nb[i]
            call("atom_rmsnorm_sh_fwd", ptr(x), N, C, ptr(b["n1w"]), ptr(b["n1b"]),
                 ptr(ws.sysn), 1e-5, ptr(nb), s)
            if ws.chunks is None:
                call("atom_rotate_in", ptr(nb), ptr(g.src), ptr(g.tgt), ptr(ws.coef), E, C,
                     ptr(ws.RAD), self.ldr, self.rad_off[i], None, ptr(ws.A1), s)
                self._gemm(ws.A1, 18 * C, E, b["so2_1"], ws.Y1[i], 11 * H, stream=s)
                self._gate_so2_2(ws, ws.Y1[i], E, b, ws.Y2[i], s)
                call("atom_rotate_back_reduce", ptr(ws.Y2[i]), ptr(ws.coef), ptr(ws.env), N, C,
                     ptr(g.recv_ptr), ptr(x), ptr(ws.xm[i]), s)
            else:
                for ch in ws.chunks:
                    self._chunk_edge_fwd(ws, i, ch, s)
                    call("atom_rotate_back_reduce", ptr(ws.Y2[0]), ptr(ws.coef[ch.e0:]),
                         ptr(ws.env[ch.e0:]), ch.n1 - ch.n0, C, ptr(ch.rp_local),
                         ptr(x[ch.n0:]), ptr(ws.xm[i][ch.n0:]), s)
            call("atom_rmsnorm_sh_fwd", ptr(ws.xm[i]), N, C, ptr(b["n2w"]), ptr(b["n2b"]), None,
                 1e-5, ptr(ws.n2), s)
            if self.ff == "grid":
                P = self.npts
                call("atom_node_project", ptr(ws.n2), N, 9, C, ptr(self.TG), P, 0, 0,
                     ptr(ws.G0), s)
                self._gemm(ws.G0, C, N * P, b["ga"], ws.h1, C, Cpre=ws.P1[i], act=1, stream=s)
                self._gemm(ws.h1, C, N * P, b["gb"], ws.h2, C, Cpre=ws.P2[i], act=1, stream=s)
                self._gemm(ws.h2, C, N * P, b["gc"], ws.h1, C, stream=s)
                ws.x[i + 1].copy_(ws.xm[i])
                call("atom_node_project", ptr(ws.h1), N, P, C, ptr(self.FG), 9, 1, 1,
                     ptr(ws.x[i + 1]), s)
            else:
                self._gemm(ws.n2, 9 * C, N, b["sm"], ws.GAT[i], 2 * H, Cpre=ws.S1[i], act=1,
                           stream=s)
                for grp in b["so3_1"]:
                    self._gemm(ws.n2, 9 * C, N, grp, ws.HS[i], 9 * H, stream=s)
                call("atom_spectral_gate_fwd", ptr(ws.HS[i]), ptr(ws.GAT[i]), N, H,
                     ptr(ws.sgg), s)
                ws.x[i + 1].copy_(ws.xm[i])
                for grp in b["so3_2"]:
                    self._gemm(ws.sgg, 9 * H, N, grp, ws.x[i + 1], 9 * C, accumulate=1,
                               stream=s)
            if i + 1 < self.NL:
                yield ("x", i + 1)
        # ---------------- final norm + energy head
        call("atom_rmsnorm_sh_fwd", ptr(ws.x[self.NL]), N, C, ptr(self.nfw), ptr(self.nfb), None,
             1e-5, ptr(ws.ne), s)
        self._gemm(ws.ne, 9 * C, N, self.eh0, ws.e1, H, Cpre=ws.e1p, act=1, stream=s)
        self._gemm(ws.e1, H, N, self.eh2, ws.e2, H, Cpre=ws.e2p, act=1, stream=s)
        self._gemm(ws.e2, H, N, self.eh4, ws.enode, 1, stream=s)
        call("atom_segment_sum", ptr(ws.enode), N, ptr(g.sys_ptr), g.nsys, ptr(ws.energy), s)
        if not forces:
            return
        yield from self._backward(ws, virial, s)

    def _backward(self, ws, virial, s):
        g = ws.graph
        N, E = g.N, g.E
        C, H, EC, NB, G, NL = self.C, self.H, self.EC, self.NB, self.G, self.NL
        P = self.npts
        ws.g_coef.zero_()
        ws.g_env.zero_()
        if ws.chunks is not None:
            ws.g_gauss.zero_()          # accumulated group by group, chunk by chunk
        # ---------------- energy head (seed dE/d e_node = 1)
        call("atom_silu_bwd", ptr(ws.eh4_rows), ptr(ws.e2p), N * H, ptr(ws.ge2), s)
        self._gemm(ws.ge2, H, N, self.eh2_bw, ws.ge1, H, stream=s)
        call("atom_silu_bwd", ptr(ws.ge1), ptr(ws.e1p), N * H, ptr(ws.ge1), s)
        ws.gne.zero_()
        self._gemm(ws.ge1, H, N, self.eh0_bw, ws.gne, 9 * C, stream=s)
        call("atom_rmsnorm_sh_bwd", ptr(ws.x[NL]), ptr(ws.gne), N, C, ptr(self.nfw), 1e-5, 0,
             ptr(ws.gx), s)
        # ---------------- blocks, reversed
        for i in reversed(range(NL)):
            b = self.blocks[i]
            if self.ff == "grid":
                # atomwise (grid) VJP
                call("atom_node_project", ptr(ws.gx), N, 9, C, ptr(self.FG), P, 0, 0,
                     ptr(ws.h1), s)
                self._gemm(ws.h1, C, N * P, b["gc_bw"], ws.h2, C, stream=s)
                call("atom_silu_bwd", ptr(ws.h2), ptr(ws.P2[i]), N * P * C, ptr(ws.h2), s)
                self._gemm(ws.h2, C, N * P, b["gb_bw"], ws.h1, C, stream=s)
                call("atom_silu_bwd", ptr(ws.h1), ptr(ws.P1[i]), N * P * C, ptr(ws.h1), s)
                self._gemm(ws.h1, C, N * P, b["ga_bw"], ws.h2, C, stream=s)
                call("atom_node_project", ptr(ws.h2), N, P, C, ptr(self.TG), 9, 1, 0,
                     ptr(ws.gn), s)
            else:
                # atomwise (spectral) VJP (tt_atom/forces.py:307-346)
                for grp in b["so3_2_bw"]:
                    self._gemm(ws.gx, 9 * C, N, grp, ws.sgg, 9 * H, stream=s)
                call("atom_spectral_gate_bwd", ptr(ws.HS[i]), ptr(ws.GAT[i]), ptr(ws.sgg), N, H,
                     ptr(ws.sgh), ptr(ws.sgat), s)
                call("atom_silu_bwd", ptr(ws.sgat), ptr(ws.S1[i]), N * 2 * H, ptr(ws.sgat), s)
                for grp in b["so3_1_bw"]:
                    self._gemm(ws.sgh, 9 * H, N, grp, ws.gn, 9 * C, stream=s)
                self._gemm(ws.sgat, 2 * H, N, b["sm_bw"], ws.gn, 9 * C, accumulate=1, stream=s)
            call("atom_rmsnorm_sh_bwd", ptr(ws.xm[i]), ptr(ws.gn), N, C, ptr(b["n2w"]), 1e-5, 1,
                 ptr(ws.gx), s)
            # edgewise VJP (gx now holds the adjoint of the block's mid point)
            if ws.chunks is not None:
                self._chunked_edge_bwd(ws, i, s)
                call("atom_rmsnorm_sh_bwd", ptr(ws.x[i]), ptr(ws.gn), N, C, ptr(b["n1w"]), 1e-5,
                     1, ptr(ws.gx), s)
                yield ("gx", i)
                continue
            call("atom_rotate_back_bwd", ptr(ws.gx), ptr(g.tgt), ptr(ws.coef), ptr(ws.env),
                 ptr(ws.Y2[i]), E, C, ptr(ws.gY2), ptr(ws.g_env), ptr(ws.g_coef), s)
            self._gemm(ws.gY2, 9 * C, E, b["so2_2_bw"], ws.Gt, 9 * H, stream=s)
            call("atom_gate_bwd", ptr(ws.Y1[i]), ptr(ws.Gt), E, H, ptr(ws.gY1), s)
            self._gemm(ws.gY1, 11 * H, E, b["so2_1_bw"], ws.A1, 18 * C, stream=s)
            # the rotated inputs are not stored: the kernel recomputes them from nb[i]
            call("atom_rotate_in_bwd_edge", ptr(ws.A1), None, ptr(ws.RAD), self.ldr,
                 self.rad_off[i], ptr(ws.nb[i]), ptr(g.src), ptr(g.tgt), ptr(ws.coef), E, C,
                 ptr(ws.grot), ptr(ws.gRAD), ptr(ws.g_coef), s)
            call("atom_rotate_in_bwd_node", ptr(ws.grot), ptr(ws.coef), N, C, ptr(g.recv_ptr),
                 ptr(g.send_ptr), ptr(g.send_eid), 0, ptr(ws.gn), s)
            call("atom_rmsnorm_sh_bwd", ptr(ws.x[i]), ptr(ws.gn), N, C, ptr(b["n1w"]), 1e-5, 1,
                 ptr(ws.gx), s)
            yield ("gx", i)
        if ws.chunks is not None:
            # edge-degree VJP and its radial group, chunk by chunk (the layers' radial groups
            # were back-propagated inside their blocks)
            for ch in ws.chunks:
                Ec = ch.e1 - ch.e0
                self._radial_group_fwd(ws, NL, ch, s)
                call("atom_edge_degree_bwd", ptr(ws.gx), ptr(g.tgt[ch.e0:]), ptr(ws.RAD),
                     ws.RAD.shape[1], ptr(ws.coef[ch.e0:]), ptr(ws.env[ch.e0:]), Ec, C, 5.0,
                     ptr(ws.gRAD), ws.gRAD.shape[1], ptr(ws.g_env[ch.e0:]),
                     ptr(ws.g_coef[ch.e0:]), s)
                self._radial_group_bwd(ws, NL, ch, s)
        else:
            self._radial_bwd_all(ws, s)
        # ---------------- geometry VJP, forces, virial
        yield from self._geometry_bwd(ws, virial, s)

    def _radial_bwd_all(self, ws, s):
        g = ws.graph
        E, C, EC, NB, G, NL = g.E, self.C, self.EC, self.NB, self.G, self.NL
        # ---------------- edge-degree VJP (gx = dE/dx_init)
        ede_off = self.rad_off[NL]
        call("atom_edge_degree_bwd", ptr(ws.gx), ptr(g.tgt), ptr(ws.RAD[:, ede_off:]), self.ldr,
             ptr(ws.coef), ptr(ws.env), E, C, 5.0, ptr(ws.gRAD[:, ede_off:]), self.ldr,
             ptr(ws.g_env), ptr(ws.g_coef), s)
        # ---------------- radial VJP (all groups), down to the Gaussian basis
        self._gemm(ws.gRAD, self.ldr, E, self.rad3_bw, ws.H2, G * EC, stream=s)
        call("atom_ln_silu_bwd", ptr(ws.R1), ptr(ws.H2), E, G * EC, G, EC, ptr(self.ln2g),
             ptr(self.ln2b), 1e-5, ptr(ws.H2), s)
        self._gemm(ws.H2, G * EC, E, self.rad2_bw, ws.H1, G * EC, stream=s)
        call("atom_ln_silu_bwd", ptr(ws.R0), ptr(ws.H1), E, G * EC, G, EC, ptr(self.ln1g),
             ptr(self.ln1b), 1e-5, ptr(ws.H1), s)
        self._gemm(ws.H1, G * EC, E, self.rad1_bw, ws.g_gauss, NB, stream=s)

    # ------------------------------------------------------- receiver-chunked edge stages
    def _radial_group_fwd(self, ws, grp, ch, s):
        """Radial function of group ``grp`` (layer grp, or the edge-degree group) for the edges
        of chunk ``ch``: R0 -> LN+SiLU -> R1 -> LN+SiLU -> ws.RAD[:Ec, :width]."""
        g, EC, NB = ws.graph, self.EC, self.NB
        rg, Ec, lo = self.radg[grp], ch.e1 - ch.e0, grp * EC
        self._gemm(ws.gauss[ch.e0:], NB, Ec, rg["r1"], ws.R0, EC, T1=self.Tsrc, T2=self.Ttgt,
                   idx1=g.zs[ch.e0:], idx2=g.zt[ch.e0:], ldt=self.G * EC, stream=s)
        call("atom_ln_silu_fwd", ptr(ws.R0), Ec, EC, 1, EC, ptr(self.ln1g[lo:]),
             ptr(self.ln1b[lo:]), 1e-5, ptr(ws.H1), s)
        self._gemm(ws.H1, EC, Ec, rg["r2"], ws.R1, EC, stream=s)
        call("atom_ln_silu_fwd", ptr(ws.R1), Ec, EC, 1, EC, ptr(self.ln2g[lo:]),
             ptr(self.ln2b[lo:]), 1e-5, ptr(ws.H2), s)
        self._gemm(ws.H2, EC, Ec, rg["r3"], ws.RAD, ws.RAD.shape[1], stream=s)

    def _radial_group_bwd(self, ws, grp, ch, s):
        """Adjoint of ``_radial_group_fwd`` (run just before, same chunk) from ws.gRAD down
        to the Gaussian basis, added into g_gauss of the chunk's edges."""
        EC, NB = self.EC, self.NB
        rg, Ec, lo = self.radg[grp], ch.e1 - ch.e0, grp * EC
        self._gemm(ws.gRAD, ws.gRAD.shape[1], Ec, rg["r3_bw"], ws.H2, EC, stream=s)
        call("atom_ln_silu_bwd", ptr(ws.R1), ptr(ws.H2), Ec, EC, 1, EC, ptr(self.ln2g[lo:]),
             ptr(self.ln2b[lo:]), 1e-5, ptr(ws.H2), s)
        self._gemm(ws.H2, EC, Ec, rg["r2_bw"], ws.H1, EC, stream=s)
        call("atom_ln_silu_bwd", ptr(ws.R0), ptr(ws.H1), Ec, EC, 1, EC, ptr(self.ln1g[lo:]),
             ptr(self.ln1b[lo:]), 1e-5, ptr(ws.H1), s)
        self._gemm(ws.H1, EC, Ec, rg["r1_bw"], ws.g_gauss[ch.e0:], NB, accumulate=1, stream=s)

    def _chunk_edge_fwd(self, ws, i, ch, s):
        """Layer i's edge chain for chunk ch up to the rotate-back input ws.Y2[0] (rows of
        the chunk's edges): radial group, rotate-in, so2_1, gate, so2_2."""
        g, C, H, b = ws.graph, self.C, self.H, self.blocks[i]
        Ec = ch.e1 - ch.e0
        self._radial_group_fwd(ws, i, ch, s)
        call("atom_rotate_in", ptr(ws.nb[i]), ptr(g.src[ch.e0:]), ptr(g.tgt[ch.e0:]),
             ptr(ws.coef[ch.e0:]), Ec, C, ptr(ws.RAD), ws.RAD.shape[1], 0, None, ptr(ws.A1), s)
        self._gemm(ws.A1, 18 * C, Ec, b["so2_1"], ws.Y1[0], 11 * H, stream=s)
        self._gate_so2_2(ws, ws.Y1[0], Ec, b, ws.Y2[0], s)

    def _chunked_edge_bwd(self, ws, i, s):
        """Edgewise VJP of layer i, chunk by chunk (each chunk's forward chain recomputed):
        ws.gx (adjoint of the block's mid point) -> ws.gn (adjoint of nb[i], accumulated over
        chunks in chunk order), and the chunk's coefficient, envelope and Gaussian adjoints."""
        g, N, C, H, b = ws.graph, ws.graph.N, self.C, self.H, self.blocks[i]
        ws.gn.zero_()
        for ch in ws.chunks:
            Ec = ch.e1 - ch.e0
            self._chunk_edge_fwd(ws, i, ch, s)
            call("atom_rotate_back_bwd", ptr(ws.gx), ptr(g.tgt[ch.e0:]), ptr(ws.coef[ch.e0:]),
                 ptr(ws.env[ch.e0:]), ptr(ws.Y2[0]), Ec, C, ptr(ws.gY2), ptr(ws.g_env[ch.e0:]),
                 ptr(ws.g_coef[ch.e0:]), s)
            self._gemm(ws.gY2, 9 * C, Ec, b["so2_2_bw"], ws.Gt, 9 * H, stream=s)
            call("atom_gate_bwd", ptr(ws.Y1[0]), ptr(ws.Gt), Ec, H, ptr(ws.gY1), s)
            self._gemm(ws.gY1, 11 * H, Ec, b["so2_1_bw"], ws.A1, 18 * C, stream=s)
            call("atom_rotate_in_bwd_edge", ptr(ws.A1), None, ptr(ws.RAD), ws.RAD.shape[1], 0,
                 ptr(ws.nb[i]), ptr(g.src[ch.e0:]), ptr(g.tgt[ch.e0:]), ptr(ws.coef[ch.e0:]),
                 Ec, C, ptr(ws.grot), ptr(ws.gRAD), ptr(ws.g_coef[ch.e0:]), s)
            call("atom_rotate_in_bwd_node", ptr(ws.grot), ptr(ws.coef[ch.e0:]), N, C,
                 ptr(ch.rp_full), ptr(ch.send_ptr), ptr(ch.send_eid), 1, ptr(ws.gn), s)
            self._radial_group_bwd(ws, i, ch, s)

    def _geometry_bwd(self, ws, virial, s):
        g = ws.graph
        N, E, NB = g.N, g.E, self.NB
        call("atom_edge_geometry_bwd", ptr(ws.pos), ptr(g.src), ptr(g.tgt), ptr(g.img),
             ptr(g.shifts), E, self.jd1, self.jd2, self.perm9, ptr(self.offset), NB, self.coeff,
             self.cutoff, ptr(ws.g_coef), ptr(ws.gauss), ptr(ws.g_gauss), ptr(ws.g_env),
             ptr(ws.g_ev), s)
        call("atom_forces_virial", ptr(ws.g_ev), ptr(ws.ev), E, N, ptr(g.recv_ptr),
             ptr(g.send_ptr), ptr(g.send_eid), ptr(ws.forces),
             ptr(ws.virial) if virial else None, ptr(ws.vscratch), s)
        yield ("forces", None)


class _Chunk:
    """One receiver chunk: nodes [n0, n1) and their received edges [e0, e1) (edges are
    receiver-major), the chunk's receiver CSR relative to e0 (local: nodes n0..n1; full: all
    N nodes, empty outside the chunk) and its sender CSR over chunk-local edge ids."""

    def __init__(self, n0, n1, e0, e1):
        self.n0, self.n1, self.e0, self.e1 = n0, n1, e0, e1


def _plan_chunks(graph, chunk_edges, stream):
    """Split the receivers into contiguous node ranges of at most ``chunk_edges`` received
    edges each (a node is never split)."""
    N = graph.N
    rp = graph.recv_ptr.long().cpu().numpy()
    dev = graph.src.device
    rp_dev = graph.recv_ptr.long()
    chunks, n0 = [], 0
    while n0 < N:
        n1 = int(np.searchsorted(rp, rp[n0] + chunk_edges, side="right")) - 1
        n1 = min(max(n1, n0 + 1), N)
        e0, e1 = int(rp[n0]), int(rp[n1])
        if e1 - e0 > chunk_edges:
            raise ValueError(f"node {n0} receives {e1 - e0} edges, more than chunk_edges "
                             f"= {chunk_edges}")
        ch = _Chunk(n0, n1, e0, e1)
        Ec = e1 - e0
        ch.rp_local = (rp_dev[n0:n1 + 1] - e0).to(torch.int32).contiguous()
        ch.rp_full = (rp_dev - e0).clamp(0, Ec).to(torch.int32).contiguous()
        ch.send_ptr = torch.empty(N + 1, dtype=torch.int32, device=dev)
        ch.send_eid = torch.empty(max(Ec, 1), dtype=torch.int32, device=dev)
        scratch = torch.empty(max(N, 1), dtype=torch.int32, device=dev)
        call("atom_sender_csr", ptr(graph.src[e0:]), Ec, N, ptr(scratch), ptr(ch.send_ptr),
             ptr(ch.send_eid), stream)
        chunks.append(ch)
        n0 = n1
    return chunks


class Workspace:
    """Every device buffer of one step for one graph topology.

    With ``chunk_edges`` the edge stages (radial function, rotate-in, SO(2) convolutions,
    gate, rotate-back and their adjoints) run over contiguous receiver chunks of at most that
    many edges, and their buffers are chunk-sized: per-edge storage is then the geometry
    (Wigner coefficients, Gaussian basis, envelope, edge vectors) and its adjoint only, and the
    reverse pass recomputes each chunk's forward chain. This is how a cell whose full per-edge
    workspace exceeds device memory runs on one GPU."""

    # device arrays of the topology; the workspace keeps its own copies at fixed addresses
    _TOPOLOGY = ("Z", "sys_id", "sys_ptr", "src", "tgt", "img", "shifts", "recv_ptr",
                 "send_ptr", "send_eid", "zs", "zt")

    def __init__(self, eng, graph, sys_emb, chunk_edges=None):
        # a graph whose arrays belong to this workspace: a same-size topology is copied into
        # them (rebind), so a step captured on these buffers stays valid
        self.graph = dataclasses.replace(
            graph, **{k: getattr(graph, k).clone() for k in self._TOPOLOGY})
        graph = self.graph
        dev = eng.device
        N, E = graph.N, graph.E
        C, H, EC, NB, G, NL = eng.C, eng.H, eng.EC, eng.NB, eng.G, eng.NL
        P = eng.npts
        f = lambda *shape: torch.empty(*shape, device=dev, dtype=torch.float32)  # noqa: E731
        self.chunk_edges = chunk_edges
        self.chunks = None
        self.pos = f(N, 3)
        # split-K scratch of node-level GEMMs (few rows): 8 splits x up to 4,096 padded rows x
        # the widest node row; larger launches have enough tiles without splitting
        self.gemm_scratch = f(8 * min(((N + 127) // 128) * 128, 4096) * 9 * max(C, H))
        self.coef, self.gauss, self.env, self.ev = f(E, 35), f(E, NB), f(E), f(E, 3)
        if chunk_edges is None:
            Eb, RW, nY, GW = E, eng.ldr, NL, G * EC
        else:
            Eb, RW, nY, GW = max(1, min(chunk_edges, E)), max(eng.radg[g]["width"]
                                                               for g in range(G)), 1, EC
        self.R0, self.H1, self.R1, self.H2 = f(Eb, GW), f(Eb, GW), f(Eb, GW), f(Eb, GW)
        self.RAD = f(Eb, RW)
        self.x = [f(N, 9, C) for _ in range(NL + 1)]
        self.nb = [f(N, 9, C) for _ in range(NL)]
        self.xm = [f(N, 9, C) for _ in range(NL)]
        self.Y1 = [f(Eb, 11 * H) for _ in range(nY)]
        self.Y2 = [f(Eb, 9 * C) for _ in range(nY)]
        self.G0 = f(N * P, C) if eng.ff == "grid" else None
        if eng.ff == "spectral":
            self.S1 = [f(N, 2 * H) for _ in range(NL)]
            self.GAT = [f(N, 2 * H) for _ in range(NL)]
            self.HS = [f(N, 9 * H) for _ in range(NL)]
            self.sgg, self.sgh, self.sgat = f(N, 9 * H), f(N, 9 * H), f(N, 2 * H)
        grid = eng.ff == "grid"
        self.P1 = [f(N * P, C) for _ in range(NL)] if grid else None
        self.P2 = [f(N * P, C) for _ in range(NL)] if grid else None
        self.A1, self.Gt = f(Eb, 18 * C), f(Eb, 9 * H)
        self.n2 = f(N, 9, C)
        self.h1, self.h2 = (f(N * P, C), f(N * P, C)) if grid else (None, None)
        self.ne, self.e1, self.e1p, self.e2, self.e2p = f(N, 9, C), f(N, H), f(N, H), f(N, H), f(N, H)
        self.enode = f(N)
        self.energy = f(graph.nsys)
        # reverse pass
        self.gY2, self.gY1, self.grot, self.gRAD = f(Eb, 9 * C), f(Eb, 11 * H), f(Eb, 18 * C), f(Eb, RW)
        self.g_coef, self.g_env, self.g_gauss, self.g_ev = f(E, 35), f(E), f(E, NB), f(E, 3)
        self.gx, self.gn, self.gne = f(N, 9, C), f(N, 9, C), f(N, 9, C)
        self.ge1, self.ge2 = f(N, H), f(N, H)
        self.eh4_rows = f(N, H)
        self.forces, self.virial, self.vscratch = f(N, 3), f(3, 3), f(9 * 1024)
        self.sysn, self.l0 = f(N, C), f(N, C)
        self._zero_sphere = torch.zeros_like(eng.sphere)
        self._eng = eng
        self.rebind(graph, sys_emb)

    def fits(self, graph):
        return (graph.N == self.graph.N and graph.E == self.graph.E
                and graph.nsys == self.graph.nsys and graph.periodic == self.graph.periodic
                and all(getattr(graph, k).shape == getattr(self.graph, k).shape
                        for k in self._TOPOLOGY))

    def rebind(self, graph, sys_emb):
        """Copy another graph of the same sizes into this workspace's topology arrays (new
        topology, same buffers and addresses) and recompute the pos-independent node
        embeddings l0 = sphere[Z] + sys_emb and the per-node system embedding."""
        assert graph.N == self.pos.shape[0]
        if graph is not self.graph:
            if not self.fits(graph):
                raise ValueError("rebind needs a graph of the workspace's sizes")
            for k in self._TOPOLOGY:
                getattr(self.graph, k).copy_(getattr(graph, k))
            self.graph.sys_ptr_host = list(graph.sys_ptr_host)
            self.graph.max_cand = max(self.graph.max_cand, graph.max_cand)
        graph = self.graph
        eng, N, eng_C = self._eng, graph.N, self._eng.C
        if self.chunk_edges is not None:
            self.chunks = _plan_chunks(graph, self.chunk_edges, L.stream_ptr())
        # energy seed: dE/d(node energy) = 1 for the atoms the energy counts (rows past the
        # last segment are a partition's halo copies and get 0)
        n_count = graph.sys_ptr_host[-1]
        self.eh4_rows[:n_count] = eng.eh4_row.reshape(1, -1)
        self.eh4_rows[n_count:] = 0
        se = sys_emb.to(eng.device, torch.float32).contiguous()    # [nsys, C]
        s = L.stream_ptr()
        call("atom_node_embed", ptr(graph.Z), ptr(graph.sys_id), ptr(self._zero_sphere), ptr(se),
             N, eng_C, ptr(self.sysn), s)
        call("atom_node_embed", ptr(graph.Z), ptr(graph.sys_id), ptr(eng.sphere), ptr(se), N,
             eng_C, ptr(self.l0), s)

    def nbytes(self):
        seen, tot = set(), 0
        for v in self.__dict__.values():
            for t in (v if isinstance(v, list) else [v]):
                if torch.is_tensor(t) and t.data_ptr() not in seen:
                    seen.add(t.data_ptr())
                    tot += t.numel() * t.element_size()
        return tot


class CapturedStep:
    """A CUDA graph of one full E+F(+virial) step on a fixed topology (the CUDA-graph
    counterpart of tt_atom/trace.py:83-215): positions are refreshed in place, then replayed."""

    def __init__(self, eng, ws, forces=True, virial=False, warmup=1, prelude=None):
        """``prelude(stream)``, when given, issues launches that run before the step inside
        the same graph (the device-resident neighbour-list refresh)."""
        self.eng, self.ws = eng, ws
        self.stream = torch.cuda.Stream(device=eng.device)
        self.stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(self.stream):
            for _ in range(warmup):
                if prelude is not None:
                    prelude(self.stream)
                eng.run(ws, ws.pos, forces=forces, virial=virial, stream=self.stream)
        torch.cuda.current_stream().wait_stream(self.stream)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=self.stream):
            if prelude is not None:
                prelude(self.stream)
            eng.run(ws, ws.pos, forces=forces, virial=virial, stream=self.stream)

    def __call__(self, pos=None):
        if pos is not None:
            self.ws.pos.copy_(pos)
        self.graph.replay()
