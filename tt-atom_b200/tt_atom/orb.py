"""Orb-v3 (conservative) energy + force + stress on the GPU, and its ASE calculator.

Reference structure (tt-atom): tt_atom/orb_model.py:127-338 (MLPNorm, Encoder,
AttentionInteractionLayer, EnergyHead), tt_atom/orb_forces.py:82-378 (their VJPs),
tt_atom/orb_geometry.py:65-139 (edge features and VJP), tt_atom/orb_calculator.py:89-215.

The edge MLP of every interaction layer is the dominant contraction. Its first linear acts on
[edges | nodes[sender] | nodes[receiver]]; here it is split: the node parts are one node-level
GEMM ``P = nodes @ [W_s; W_r]^T`` ([N, 2 hidden]) whose rows are gathered and added in the edge
GEMM's epilogue, so the gathered [E, 3C] input is never built (K drops from 3C to C). Its
reverse pass likewise sums the first-layer adjoint per node (CSR) before one node-level GEMM.
SiLU is fused into the GEMM epilogues (pre-activations kept for the reverse pass); RMSNorm and
the residual update are one kernel.

Not on the GPU: the energy normaliser / per-element references (a few scalars applied on the
host when the weights carry them). The ZBL pair repulsion runs on the GPU (``atom_orb_zbl``).
"""
from __future__ import annotations

import dataclasses

import numpy as np
import torch

from . import _lib as L
from ._lib import ptr
from .ase_compat import _AseCalculator, all_changes, atoms_volume, voigt_6
from .engine import (PRECISIONS, CapturedStep, Workspace, _Groups, _dev, call, to_host,
                     upload_positions)
from .graph import build_graph


class OrbEngine:
    def __init__(self, weights, cfg, device="cuda", precision="3xtf32"):
        L.lib()
        self.device = torch.device(device)
        self.cfg = dict(cfg)
        self.precision = PRECISIONS[precision]
        C, Hd = cfg["latent_dim"], cfg["hidden_dim"]
        self.C, self.Hd, self.NL = C, Hd, cfg["num_message_passing_steps"]
        self.nb, self.rmax = cfg["num_bases"], float(cfg["cutoff"])
        self.D0 = cfg["node_embed_size"]
        w = {k: v.float() for k, v in weights.items()}
        d = lambda t: _dev(t, self.device)  # noqa: E731

        def lin_groups(W, b=None, a_col=0, c_col=0):
            return _Groups([dict(a_col=a_col, K=W.shape[1], c_col=c_col, N=W.shape[0],
                                 B=d(W.t()), bias=b)])

        def bw_groups(W):       # g_in = g_out @ W
            return _Groups([dict(a_col=0, K=W.shape[0], c_col=0, N=W.shape[1], B=d(W))])

        def mlpnorm(p):
            (W0, b0), (W1, b1), (W2, b2) = [(w[f"{p}.mlp.NN-{i}.weight"],
                                            w[f"{p}.mlp.NN-{i}.bias"]) for i in range(3)]
            return dict(f0=lin_groups(W0, d(b0)), f1=lin_groups(W1, d(b1)),
                        f2=lin_groups(W2, d(b2)), b0=bw_groups(W0), b1=bw_groups(W1),
                        b2=bw_groups(W2), nw=d(w[f"{p}.layer_norm.weight"]), W0=W0, b0v=d(b0))

        self.emb = d(w["atom_emb.embeddings.weight"])
        self.zero_row = torch.zeros(1, self.D0, device=self.device)
        # OrbMol checkpoints condition on the system's charge and spin: a fixed embedding,
        # projected per layer and added to the nodes at the layer's start
        # (tt_atom/orb_model.py:32-57, 219-237); the host keeps the small weights
        self.has_cond = "conditioner.charge_embedding.W" in w
        if self.has_cond:
            self.cond_w = (w["conditioner.charge_embedding.W"].double(),
                           w["conditioner.spin_embedding.W"].double())
            self.cond_proj = [(w[f"gnn_stacks.{i}._cond_node_proj.weight"].double(),
                               w[f"gnn_stacks.{i}._cond_node_proj.bias"].double())
                              for i in range(self.NL)]
        self.enc_n = mlpnorm("_encoder._node_fn")
        self.enc_e = mlpnorm("_encoder._edge_fn")
        self.layers = []
        for i in range(self.NL):
            p = f"gnn_stacks.{i}"
            em, nm = mlpnorm(f"{p}._edge_mlp"), mlpnorm(f"{p}._node_mlp")
            W0 = em["W0"]                               # [Hd, 3C]: edges | sender | receiver
            Wa, Ws, Wr = W0[:, :C], W0[:, C:2 * C], W0[:, 2 * C:]
            em["f0"] = _Groups([dict(a_col=0, K=C, c_col=0, N=Hd, B=d(Wa.t()), bias=em["b0v"])])
            em["proj"] = _Groups([dict(a_col=0, K=C, c_col=0, N=Hd, B=d(Ws.t())),
                                  dict(a_col=0, K=C, c_col=Hd, N=Hd, B=d(Wr.t()))])
            em["b0a"] = _Groups([dict(a_col=0, K=Hd, c_col=0, N=C, B=d(Wa))])
            em["b0sr"] = _Groups([dict(a_col=0, K=2 * Hd, c_col=0, N=C,
                                       B=d(torch.cat([Ws, Wr], 0)))])
            nW0 = nm["W0"]
            nm["b0n"] = _Groups([dict(a_col=0, K=Hd, c_col=0, N=C, B=d(nW0[:, :C]))])
            nm["b0agg"] = _Groups([dict(a_col=0, K=Hd, c_col=0, N=2 * C, B=d(nW0[:, C:]))])
            self.layers.append(dict(
                em=em, nm=nm,
                wr=d(w[f"{p}._receive_attn.weight"].reshape(-1)),
                br=float(w[f"{p}._receive_attn.bias"].reshape(-1)[0]),
                ws=d(w[f"{p}._send_attn.weight"].reshape(-1)),
                bs=float(w[f"{p}._send_attn.bias"].reshape(-1)[0])))
        H0, Hb0 = w["energy_head.mlp.NN-0.weight"], w["energy_head.mlp.NN-0.bias"]
        H1, Hb1 = w["energy_head.mlp.NN-1.weight"], w["energy_head.mlp.NN-1.bias"]
        self.hh = H0.shape[0]
        self.head0 = lin_groups(H0, d(Hb0))
        self.head1 = lin_groups(H1, d(Hb1))
        self.head1_row = d(H1.reshape(-1))
        self.head0_bw = bw_groups(H0)
        # direct checkpoints (orb-v3-direct-*): per-node force head and node-mean stress head
        self.direct = "forces_head.mlp.NN-0.weight" in w
        self.has_stress_head = "stress_head.mlp.NN-0.weight" in w
        if self.direct:
            F0, F1 = w["forces_head.mlp.NN-0.weight"], w["forces_head.mlp.NN-1.weight"]
            self.fh = F0.shape[0]
            self.fhead0 = lin_groups(F0, d(w["forces_head.mlp.NN-0.bias"]))
            self.fhead1 = lin_groups(F1, d(w["forces_head.mlp.NN-1.bias"]))
        if self.has_stress_head:
            S0, S1 = w["stress_head.mlp.NN-0.weight"], w["stress_head.mlp.NN-1.weight"]
            self.sh = S0.shape[0]
            self.shead0 = lin_groups(S0, d(w["stress_head.mlp.NN-0.bias"]))
            self.shead1 = lin_groups(S1, d(w["stress_head.mlp.NN-1.bias"]))

    def _gemm(self, A, lda, M, groups, Cout, ldc, *, Cpre=None, T1=None, T2=None, idx1=None,
              idx2=None, ldt=0, act=0, accumulate=0, s=0):
        # the workspace's scratch lets node-level launches (few rows) split K over more CTAs
        sc = self._scratch
        if self.precision == 3:
            groups.ensure_f16()
        call("atom_gemm_ex", ptr(A), lda, M, groups.struct, ptr(Cout), ldc, ptr(Cpre), ptr(T1),
             ptr(T2), ptr(idx1), ptr(idx2), ldt, act, accumulate, self.precision, ptr(sc),
             sc.numel() if sc is not None else 0, s)

    def workspace(self, graph):
        return OrbWorkspace(self, graph)

    def set_condition(self, ws, charge=0.0, spin=0.0):
        """Per-layer conditioning rows of a system's total charge and spin into ``ws.cond``
        (outside any captured step, which reads them from there): [sin, cos] of value * W *
        2 pi for each, a zero spin giving zeros, projected by each layer's node projection."""
        if not self.has_cond:
            return
        c = charge_spin_embedding(self.cond_w[0], self.cond_w[1], charge, spin)
        rows = torch.stack([W @ c + b for W, b in self.cond_proj]).float()
        ws.cond.copy_(rows)

    # ---------------------------------------------------------------------------- forward
    def _mlpnorm_fwd(self, m, X, ldx, M, a0, a1, h2, tmp0, tmp1, s, first=None):
        Hd = self.Hd
        if first is None:
            self._gemm(X, ldx, M, m["f0"], tmp0, Hd, Cpre=a0, act=1, s=s)
        else:
            first(tmp0, a0)
        self._gemm(tmp0, Hd, M, m["f1"], tmp1, Hd, Cpre=a1, act=1, s=s)
        self._gemm(tmp1, Hd, M, m["f2"], h2, self.C, s=s)

    def launches_per_step(self, ws, forces=True, virial=True):
        """Number of this library's kernels one ``run`` launches (the library's own counter)."""
        from .engine import launch_count
        torch.cuda.synchronize()
        c0 = launch_count()
        self.run(ws, forces=forces, virial=virial)
        torch.cuda.synchronize()
        return launch_count() - c0

    def time_kernels(self, ws, reps=5):
        """Device time of the dominant kernel: the layer-0 edge-MLP hidden GEMM
        ([E, hidden] x [hidden, hidden], SiLU epilogue), timed with CUDA events on its stream."""
        st = torch.cuda.Stream(device=self.device)
        st.wait_stream(torch.cuda.current_stream())
        E, Hd = ws.graph.E, self.Hd
        em = self.layers[0]["em"]
        with torch.cuda.stream(st):
            s = st.cuda_stream
            self._gemm(ws.et0, Hd, E, em["f1"], ws.et1, Hd, Cpre=ws.ea1[0], act=1, s=s)
            t0 = torch.cuda.Event(enable_timing=True)
            t1 = torch.cuda.Event(enable_timing=True)
            t0.record(st)
            for _ in range(reps):
                self._gemm(ws.et0, Hd, E, em["f1"], ws.et1, Hd, Cpre=ws.ea1[0], act=1, s=s)
            t1.record(st)
        st.synchronize()
        torch.cuda.current_stream().wait_stream(st)
        return dict(name="Orb edge-MLP hidden GEMM", ms=t0.elapsed_time(t1) / reps,
                    flop=2.0 * E * Hd * Hd)

    _scratch = None

    def run(self, ws, pos=None, forces=True, virial=False, stream=None):
        """One E (+F, +virial) evaluation on ``ws``'s graph (``pos`` defaults to ws.pos)."""
        self._scratch = ws.gemm_scratch
        if pos is not None and pos.data_ptr() != ws.pos.data_ptr():
            ws.pos.copy_(pos)
        s = L.stream_ptr(stream)
        g = ws.graph
        N, E, C, Hd = g.N, g.E, self.C, self.Hd
        C3 = 3 * C
        call("atom_orb_edge_features", ptr(ws.pos), ptr(g.src), ptr(g.tgt), ptr(g.img),
             ptr(g.shifts), E, self.rmax, self.nb, ptr(ws.feat), ptr(ws.cut), ptr(ws.ev), s)
        # encoder: node features -> node_in[0][:, :C]; edge features -> edges[0]
        self._mlpnorm_fwd(self.enc_n, ws.x0, self.D0, N, ws.na0[-1], ws.na1[-1], ws.nh2[-1],
                          ws.nt0, ws.nt1, s)
        call("atom_rmsnorm_rows", ptr(ws.nh2[-1]), C, N, C, ptr(self.enc_n["nw"]), 1e-6,
             ptr(ws.node_in[0]), C3, None, 0, None, 0, s)
        self._mlpnorm_fwd(self.enc_e, ws.feat, 16 * self.nb, E, ws.ea0[-1], ws.ea1[-1],
                          ws.eh2[-1], ws.et0, ws.et1, s)
        call("atom_rmsnorm_rows", ptr(ws.eh2[-1]), C, E, C, ptr(self.enc_e["nw"]), 1e-6,
             ptr(ws.edges[0]), C, None, 0, None, 0, s)
        for i, lay in enumerate(self.layers):
            nodes, edges = ws.node_in[i], ws.edges[i]
            if self.has_cond:           # the layer's input nodes += its conditioning row
                call("atom_row_broadcast", ptr(ws.cond[i]), N, C, 1.0, ptr(nodes), C3, 1, s)
            call("atom_orb_attention", ptr(edges), E, C, ptr(lay["wr"]), lay["br"],
                 ptr(lay["ws"]), lay["bs"], ptr(ws.cut), ptr(ws.lin[i]), ptr(ws.att[i]), s)
            em, nm = lay["em"], lay["nm"]
            # node projections for the gathered part of the edge MLP's first linear
            self._gemm(nodes, C3, N, em["proj"], ws.P, 2 * Hd, s=s)

            def first(out, pre, em=em, edges=edges):
                self._gemm(edges, C, E, em["f0"], out, Hd, Cpre=pre, T1=ws.P, T2=ws.P[:, Hd:],
                           idx1=g.tgt, idx2=g.src, ldt=2 * Hd, act=1, s=s)
            self._mlpnorm_fwd(em, None, 0, E, ws.ea0[i], ws.ea1[i], ws.eh2[i], ws.et0, ws.et1, s,
                              first=first)
            # ue = RMSNorm(h2); edges[i+1] = edges[i] + ue
            call("atom_rmsnorm_rows", ptr(ws.eh2[i]), C, E, C, ptr(em["nw"]), 1e-6,
                 ptr(ws.ue[i]), C, ptr(edges), C, ptr(ws.edges[i + 1]), C, s)
            # aggregates into node_in[i][:, C:3C]: receivers (= src) then senders (= tgt)
            call("atom_csr_sum", ptr(ws.ue[i]), C, ptr(ws.att[i]), 2, ptr(g.send_ptr),
                 ptr(g.send_eid), N, C, ptr(nodes[:, C:]), C3, 0, s)
            call("atom_csr_sum", ptr(ws.ue[i]), C, ptr(ws.att[i][:, 1:]), 2, ptr(g.recv_ptr),
                 None, N, C, ptr(nodes[:, 2 * C:]), C3, 0, s)
            self._mlpnorm_fwd(nm, nodes, C3, N, ws.na0[i], ws.na1[i], ws.nh2[i], ws.nt0, ws.nt1,
                              s)
            call("atom_rmsnorm_rows", ptr(ws.nh2[i]), C, N, C, ptr(nm["nw"]), 1e-6, None, 0,
                 ptr(nodes), C3, ptr(ws.node_in[i + 1]), C3, s)
        # energy head on the node mean
        call("atom_col_mean", ptr(ws.node_in[self.NL]), C3, N, C, 1.0 / N, ptr(ws.mean), s)
        self._gemm(ws.mean, C, 1, self.head0, ws.hh, self.hh, Cpre=ws.hhp, act=1, s=s)
        self._gemm(ws.hh, self.hh, 1, self.head1, ws.energy, 1, s=s)
        if forces:
            self._backward(ws, virial, s)

    def direct_heads(self, ws, stress=False, stream=None):
        """Direct checkpoints, after a forward ``run(ws, forces=False)``: raw (normalised
        space) per-atom forces with the net force removed -> ws.fraw[:, :3]
        (tt_atom/orb_model.py:358-388) and the raw Voigt-6 stress of the node mean -> ws.sraw
        (tt_atom/orb_model.py:407-436)."""
        s = L.stream_ptr(stream)
        N, C = ws.graph.N, self.C
        nodes = ws.node_in[self.NL]                     # [N, 3C], latent in the first C
        self._gemm(nodes, 3 * C, N, self.fhead0, ws.fhid, self.fh, act=1, s=s)
        self._gemm(ws.fhid, self.fh, N, self.fhead1, ws.fraw, 4, s=s)
        call("atom_col_mean", ptr(ws.fraw), 4, N, 4, 1.0 / N, ptr(ws.fmean), s)
        call("atom_row_broadcast", ptr(ws.fmean), N, 4, -1.0, ptr(ws.fraw), 4, 1, s)
        if stress:
            if not self.has_stress_head:
                raise ValueError("stress requested but this direct checkpoint carries no "
                                 "stress_head weights")
            self._gemm(ws.mean, C, 1, self.shead0, ws.shid, self.sh, act=1, s=s)
            self._gemm(ws.shid, self.sh, 1, self.shead1, ws.sraw, 8, s=s)

    # --------------------------------------------------------------------------- reverse
    def _mlpnorm_bwd(self, m, h2, gY, M, a0, a1, tmp0, tmp1, g_a0, s):
        """gY: adjoint of the normalised output [M, C] (overwritten with the h2 adjoint);
        returns the first layer's pre-activation adjoint in g_a0 [M, Hd]."""
        C, Hd = self.C, self.Hd
        call("atom_rmsnorm_rows_bwd", ptr(h2), ptr(gY), M, C, ptr(m["nw"]), 1e-6, ptr(gY), s)
        self._gemm(gY, C, M, m["b2"], tmp1, Hd, s=s)
        call("atom_silu_bwd", ptr(tmp1), ptr(a1), M * Hd, ptr(tmp1), s)
        self._gemm(tmp1, Hd, M, m["b1"], tmp0, Hd, s=s)
        call("atom_silu_bwd", ptr(tmp0), ptr(a0), M * Hd, ptr(g_a0), s)

    def _backward(self, ws, virial, s):
        g = ws.graph
        N, E, C, Hd = g.N, g.E, self.C, self.Hd
        ws.g_cut.zero_()
        # head: dE/dmean, broadcast / N to every node
        call("atom_silu_bwd", ptr(self.head1_row), ptr(ws.hhp), self.hh, ptr(ws.ghh), s)
        self._gemm(ws.ghh, self.hh, 1, self.head0_bw, ws.gmean, C, s=s)
        call("atom_row_broadcast", ptr(ws.gmean), N, C, 1.0 / N, ptr(ws.gN), C, 0, s)
        ws.gE.zero_()
        for i in reversed(range(self.NL)):
            lay = self.layers[i]
            em, nm = lay["em"], lay["nm"]
            # node MLP: its output adds to nodes -> adjoint gN
            ws.gtmpN.copy_(ws.gN)
            self._mlpnorm_bwd(nm, ws.nh2[i], ws.gtmpN, N, ws.na0[i], ws.na1[i], ws.nt0, ws.nt1,
                              ws.nt0, s)
            self._gemm(ws.nt0, Hd, N, nm["b0n"], ws.gN, C, accumulate=1, s=s)
            self._gemm(ws.nt0, Hd, N, nm["b0agg"], ws.gagg, 2 * C, s=s)
            # aggregates + attention gates -> g_ue, gE (+gate part), g_cut
            call("atom_orb_messages_bwd", ptr(ws.gagg), ptr(ws.gE), ptr(ws.ue[i]),
                 ptr(ws.lin[i]), ptr(ws.att[i]), ptr(ws.cut), ptr(g.src), ptr(g.tgt), E, C,
                 ptr(lay["wr"]), ptr(lay["ws"]), ptr(ws.gue), ptr(ws.gE), ptr(ws.g_cut), s)
            # edge MLP
            self._mlpnorm_bwd(em, ws.eh2[i], ws.gue, E, ws.ea0[i], ws.ea1[i], ws.et0, ws.et1,
                              ws.et0, s)
            self._gemm(ws.et0, Hd, E, em["b0a"], ws.gE, C, accumulate=1, s=s)
            call("atom_csr_sum", ptr(ws.et0), Hd, None, 0, ptr(g.recv_ptr), None, N, Hd,
                 ptr(ws.gP), 2 * Hd, 0, s)
            call("atom_csr_sum", ptr(ws.et0), Hd, None, 0, ptr(g.send_ptr), ptr(g.send_eid), N,
                 Hd, ptr(ws.gP[:, Hd:]), 2 * Hd, 0, s)
            self._gemm(ws.gP, 2 * Hd, N, em["b0sr"], ws.gN, C, accumulate=1, s=s)
        # edge encoder -> edge-feature adjoint
        self._mlpnorm_bwd(self.enc_e, ws.eh2[-1], ws.gE, E, ws.ea0[-1], ws.ea1[-1], ws.et0,
                          ws.et1, ws.et0, s)
        self._gemm(ws.et0, Hd, E, self.enc_e["b0"], ws.gfeat, 16 * self.nb, s=s)
        call("atom_orb_edge_features_bwd", ptr(ws.pos), ptr(g.src), ptr(g.tgt), ptr(g.img),
             ptr(g.shifts), E, self.rmax, self.nb, ptr(ws.gfeat), ptr(ws.g_cut), ptr(ws.g_ev), s)
        call("atom_forces_virial", ptr(ws.g_ev), ptr(ws.ev), E, N, ptr(g.recv_ptr),
             ptr(g.send_ptr), ptr(g.send_eid), ptr(ws.forces),
             ptr(ws.virial) if virial else None, ptr(ws.vscratch), s)


class OrbWorkspace:
    _TOPOLOGY = Workspace._TOPOLOGY

    def __init__(self, eng, graph):
        # the workspace's own topology arrays (fixed addresses: a captured step stays valid
        # when a same-size edge set is copied in)
        self.graph = dataclasses.replace(
            graph, **{k: getattr(graph, k).clone() for k in self._TOPOLOGY})
        graph = self.graph
        dev = eng.device
        N, E, C, Hd, NL = graph.N, graph.E, eng.C, eng.Hd, eng.NL
        f = lambda *sh: torch.empty(*sh, device=dev, dtype=torch.float32)  # noqa: E731
        self.pos = f(N, 3)
        # split-K scratch of node-level GEMMs: 8 splits x padded rows x the widest node row
        self.gemm_scratch = f(8 * ((N + 127) // 128) * 128 * max(2 * Hd, 3 * C))
        self.feat, self.cut, self.ev = f(E, 16 * eng.nb), f(E), f(E, 3)
        self.x0 = f(N, eng.D0)
        self.cond = torch.zeros(eng.NL, eng.C, device=dev)      # conditioning rows per layer
        self._eng = eng
        self.rebind(graph)
        # per layer (+1 slot at the end for the encoder)
        self.ea0 = [f(E, Hd) for _ in range(NL + 1)]
        self.ea1 = [f(E, Hd) for _ in range(NL + 1)]
        self.eh2 = [f(E, C) for _ in range(NL + 1)]
        self.na0 = [f(N, Hd) for _ in range(NL + 1)]
        self.na1 = [f(N, Hd) for _ in range(NL + 1)]
        self.nh2 = [f(N, C) for _ in range(NL + 1)]
        self.ue = [f(E, C) for _ in range(NL)]
        self.lin = [f(E, 2) for _ in range(NL)]
        self.att = [f(E, 2) for _ in range(NL)]
        self.edges = [f(E, C) for _ in range(NL + 1)]
        self.node_in = [f(N, 3 * C) for _ in range(NL + 1)]
        self.et0, self.et1 = f(E, Hd), f(E, Hd)
        self.nt0, self.nt1 = f(N, Hd), f(N, Hd)
        self.P = f(N, 2 * Hd)
        self.mean, self.hh, self.hhp = f(1, C), f(1, eng.hh), f(1, eng.hh)
        if eng.direct:
            self.fhid, self.fraw, self.fmean = f(N, eng.fh), torch.zeros(N, 4, device=dev), f(4)
        if eng.has_stress_head:
            self.shid, self.sraw = f(1, eng.sh), torch.zeros(1, 8, device=dev)
        self.energy = f(1)
        self.ghh, self.gmean = f(1, eng.hh), f(1, C)
        self.gN, self.gtmpN, self.gagg = f(N, C), f(N, C), f(N, 2 * C)
        self.gE, self.gue, self.gP = f(E, C), f(E, C), f(N, 2 * Hd)
        self.gfeat, self.g_cut, self.g_ev = f(E, 16 * eng.nb), f(E), f(E, 3)
        self.forces, self.virial, self.vscratch = f(N, 3), f(3, 3), f(9 * 1024)


    def nbytes(self):
        from .engine import Workspace
        return Workspace.nbytes(self)

    def fits(self, graph):
        return Workspace.fits(self, graph)

    def rebind(self, graph):
        """Copy a graph of the same sizes into the workspace's topology arrays; recompute the
        node input rows (the species embedding lookup)."""
        if graph is not self.graph:
            if not self.fits(graph):
                raise ValueError("rebind needs a graph of the workspace's sizes")
            for k in self._TOPOLOGY:
                getattr(self.graph, k).copy_(getattr(graph, k))
            self.graph.sys_ptr_host = list(graph.sys_ptr_host)
            self.graph.max_cand = max(self.graph.max_cand, graph.max_cand)
        graph = self.graph
        eng = self._eng
        call("atom_node_embed", ptr(graph.Z), None, ptr(eng.emb), ptr(eng.zero_row), graph.N,
             eng.D0, ptr(self.x0), L.stream_ptr())


# Covalent radii (Angstrom) indexed by atomic number, Cordero et al., Dalton Trans. 2008,
# 2832-2838 (low-spin values for Mn, Fe, Co; sp3 carbon), the table ASE ships as
# ase.data.covalent_radii (index 0 and elements past Cm: 0.2). The reference's ZBL term looks
# it up at Z + 1 (tt_atom/orb_model.py:507-523).
COVALENT_RADII = (
    0.20, 0.31, 0.28, 1.28, 0.96, 0.84, 0.76, 0.71, 0.66, 0.57, 0.58, 1.66, 1.41, 1.21, 1.11,
    1.07, 1.05, 1.02, 1.06, 2.03, 1.76, 1.70, 1.60, 1.53, 1.39, 1.39, 1.32, 1.26, 1.24, 1.32,
    1.22, 1.22, 1.20, 1.19, 1.20, 1.20, 1.16, 2.20, 1.95, 1.90, 1.75, 1.64, 1.54, 1.47, 1.46,
    1.42, 1.39, 1.45, 1.44, 1.42, 1.39, 1.39, 1.38, 1.39, 1.40, 2.44, 2.15, 2.07, 2.04, 2.03,
    2.01, 1.99, 1.98, 1.98, 1.96, 1.94, 1.92, 1.92, 1.89, 1.90, 1.87, 1.87, 1.75, 1.70, 1.62,
    1.51, 1.44, 1.41, 1.36, 1.36, 1.32, 1.45, 1.46, 1.48, 1.40, 1.50, 1.50, 2.60, 2.21, 2.15,
    2.06, 2.00, 1.96, 1.90, 1.87, 1.80, 1.69) + (0.20,) * 22


def charge_spin_embedding(charge_W, spin_W, charge, spin):
    """OrbMol's charge / spin conditioning vector (tt_atom/orb_model.py:32-56): [sin, cos] of
    value * W * 2 pi for the charge and for the spin, a zero spin giving zeros."""
    import math

    def emb(v, W, is_spin):
        x = float(v) * W * 2.0 * math.pi
        e = torch.cat([torch.sin(x), torch.cos(x)])
        return torch.zeros_like(e) if is_spin and v == 0 else e
    return torch.cat([emb(charge, charge_W, False), emb(spin, spin_W, True)])


def _affine(x, weights, prefix):
    """A scalar normaliser's inverse, x * sqrt(running_var) + running_mean (identity when the
    weights carry no such normaliser)."""
    var = weights.get(f"{prefix}.running_var")
    if var is None:
        return x
    mu = weights.get(f"{prefix}.running_mean")
    return x * float(var.double().sqrt()) + (float(mu) if mu is not None else 0.0)


def force_denormalize(raw, weights):
    """Direct checkpoints' force head normaliser (tt_atom/orb_model.py:438-442)."""
    return _affine(raw, weights, "forces_head.normalizer.bn")


def stress_denormalize(raw, weights):
    """Direct checkpoints' stress head normalisers, diagonal and off-diagonal Voigt components
    each through their own (tt_atom/orb_model.py:445-456)."""
    return torch.cat([_affine(raw[:3], weights, "stress_head.diag_normalizer.bn"),
                      _affine(raw[3:], weights, "stress_head.offdiag_normalizer.bn")])


def conservative_scale(weights, n):
    """Conservative checkpoints: forces and virial of the raw energy times sigma * n, the only
    factor of the energy normaliser that survives differentiation (tt_atom/orb_model.py:459-488);
    1 without a normaliser."""
    var = weights.get("energy_head.normalizer.bn.running_var")
    return 1.0 if var is None else float(var.double().sqrt()) * n


def conservative_stress(virial, n, cell, weights):
    """Voigt-6 stress of a conservative checkpoint from its raw virial: scaled by sigma * n,
    divided by the cell volume, off-diagonal pairs averaged (tt_atom/orb_model.py:472-488)."""
    vol = abs(float(np.linalg.det(np.asarray(cell, dtype=np.float64))))
    return voigt_6(conservative_scale(weights, n) * np.asarray(virial, dtype=np.float64) / vol)


def energy_denormalize(raw, Z, weights):
    """The energy head's normaliser (tt_atom/orb_model.py:590-600, ``EnergyHead.denormalize``):
    undo the scalar normaliser's affine (running mean / variance), undo the per-atom average
    (times the atom count) and add the per-element linear reference energies. ``raw`` may be a
    Python float or a (device) tensor; weights without a normaliser return ``raw`` unchanged."""
    w = weights
    if "energy_head.normalizer.bn.running_var" not in w:
        return raw
    sigma = float(w["energy_head.normalizer.bn.running_var"].double().sqrt())
    mean = float(w["energy_head.normalizer.bn.running_mean"])
    Z = np.asarray(Z, dtype=np.int64)
    ref = float(w["energy_head.reference.linear.weight"].double().reshape(-1)[Z].sum())
    return (raw * sigma + mean) * len(Z) + ref


class OrbCalculator(_AseCalculator):
    """ASE calculator for Orb-v3 conservative bundles (tt_atom/orb_calculator.py:28-215):
    energy, forces = -dE/dpos and stress from the strain virial. Energies are the raw model
    output, denormalised on the host when the weights carry ``energy_head.normalizer`` /
    ``energy_head.reference`` entries, plus (``zbl=True``, the reference's behaviour) the ZBL
    pair repulsion computed on the GPU (``atom_orb_zbl``, per-node mean)."""

    implemented_properties = ["energy", "free_energy", "energies", "forces", "stress"]

    def __init__(self, weights, device=None, device_id=0, fast=False, bucketing=False, *,
                 cfg=None, precision="3xtf32", max_num_neighbors="config", zbl=True,
                 trace=False, **kwargs):
        """The reference's signature (tt_atom/orb_calculator.py:26): ``weights`` a bundle (or its
        path) or, with ``cfg``, a weight dict. ``fast`` and ``bucketing`` are accepted for
        compatibility: they select device compile and padding policies of the reference that have
        no counterpart here (edge counts need no padding to shape buckets on this GPU, and
        results are the same)."""
        super().__init__(**kwargs)
        self.zbl = zbl
        # trace: the model pass is captured as a CUDA graph and replayed (also after the edge
        # set changes, as long as its sizes do not), like TTAtomCalculator(trace=True)
        self.trace = trace
        self._step = self._step_key = None
        if cfg is None:
            from .weights import WeightBundle
            b = WeightBundle.load(weights) if isinstance(weights, str) else weights
            cfg, weights = b.config, b.weights
        self.cfg = cfg
        self._w = weights
        self.device = torch.device(device) if device is not None else torch.device("cuda",
                                                                                    device_id)
        self.engine = OrbEngine(weights, cfg, self.device, precision)
        self.max_nbrs = cfg.get("max_num_neighbors") if max_num_neighbors == "config" \
            else max_num_neighbors
        self._ws = None
        self._rcov = torch.tensor(COVALENT_RADII, dtype=torch.float64, device=self.device)

    @classmethod
    def from_checkpoint(cls, checkpoint="orb-v3-conservative-inf-omat", refenv=None,
                        cache_dir=None, device=None, device_id=0, fast=False, **kwargs):
        """A calculator for a released Orb-v3 checkpoint from its cached exported weights
        (tt_atom/orb_calculator.py:75-87). A cache miss raises: exporting the weights needs the
        reference environment, which this build does not include."""
        from . import bundle_cache as BC
        from .weights import WeightBundle
        path = BC.cached(BC.orb_weights_path(checkpoint, cache_dir), f"{checkpoint} weights")
        return cls(WeightBundle.load(path), device=device, device_id=device_id, **kwargs)

    def _zbl(self, ws, stress, scale=None):
        """ZBL energy (``scale`` times the pair sum: 1 / N, the per-node mean, by default),
        forces and virial on ``ws``'s graph (its edge vectors ``ws.ev`` are those of the last
        ``engine.run``), as host values."""
        E, F, V = to_host(*self._zbl_launch(ws, stress, scale))
        return float(E[0]), F, V

    def _zbl_launch(self, ws, stress, scale=None):
        """Launch the ZBL term (see ``_zbl``); returns its device tensors (energy [1] float64,
        forces [N, 3], virial [3, 3] or None)."""
        g, N, E = ws.graph, ws.graph.N, ws.graph.E
        if getattr(ws, "zbl_gev", None) is None or ws.zbl_gev.shape[0] != max(E, 1):
            f = lambda *sh, dt=torch.float32: torch.empty(*sh, device=self.device, dtype=dt)  # noqa: E731
            ws.zbl_gev, ws.zbl_F, ws.zbl_V = f(max(E, 1), 3), f(N, 3), f(3, 3)
            ws.zbl_part = f(1024, dt=torch.float64)
            ws.zbl_E = f(1, dt=torch.float64)
        s = L.stream_ptr()
        call("atom_orb_zbl", ptr(ws.ev), ptr(g.Z), ptr(g.src), ptr(g.tgt), E, ptr(self._rcov),
             len(COVALENT_RADII), 1.0 / N if scale is None else scale, ptr(ws.zbl_gev),
             ptr(ws.zbl_part), ptr(ws.zbl_E), s)
        call("atom_forces_virial", ptr(ws.zbl_gev), ptr(ws.ev), E, N, ptr(g.recv_ptr),
             ptr(g.send_ptr), ptr(g.send_eid), ptr(ws.zbl_F),
             ptr(ws.zbl_V) if stress else None, ptr(ws.vscratch), s)
        return ws.zbl_E, ws.zbl_F, (ws.zbl_V if stress else None)

    def _evaluate_direct(self, pos, Z, cell, pbc, stress=False, charge=0.0, spin=0.0):
        """Direct checkpoints: raw energy, raw per-atom forces [N, 3] (net force removed) and
        raw Voigt-6 stress (or None) from one forward pass and the heads."""
        self._evaluate(pos, Z, cell, pbc, forces=False, stress=False, charge=charge, spin=spin)
        ws = self._ws
        self.engine.direct_heads(ws, stress=stress)
        E = float(ws.energy.double().cpu()[0])
        F = ws.fraw[:, :3].double().cpu()
        S = ws.sraw[0, :6].double().cpu() if stress else None
        return E, F, S

    def _system_key(self, Z, cell, pbc, forces, stress, charge, spin):
        Z = np.asarray(Z, dtype=np.int64)
        return (Z.shape[0], Z.tobytes(),
                None if cell is None else np.asarray(cell, np.float32).tobytes(),
                None if pbc is None else tuple(np.broadcast_to(np.asarray(pbc, bool), 3)),
                bool(forces), bool(stress), float(charge), float(spin))

    def _refresh_step(self, pos, key, forces, stress, device_out, defer_status=False):
        """Traced evaluation of the previous call's system at new positions: one captured graph
        rebuilds the neighbour list on the device and runs the model pass (see
        TTAtomCalculator); None when it does not apply or the edge count changed."""
        from .graph import TopologyRefresh
        ws = self._ws
        if ws is None or getattr(self, "_refresh_key", None) != key:
            return None
        full = getattr(self, "_full_step", None)
        upload_positions(ws, pos)
        if full is None or full[0] is not ws:
            refresh = TopologyRefresh(ws.graph)
            step = CapturedStep(self.engine, ws, forces=forces, virial=stress,
                                prelude=lambda st: refresh.launch(ws.pos, st))
            self._full_step = full = (ws, refresh, step)
        _, refresh, step = full
        step()
        if device_out:
            if defer_status:
                # the caller reads the status with its results (one read-back) and calls
                # refresh_failed() when it is not OK
                self._pending_status = refresh.status[:1]
                return ws.energy, ws.forces, (ws.virial if stress else None)
            if int(refresh.status[0]) != TopologyRefresh.OK:
                self._refresh_key = self._full_step = None
                return None
            return ws.energy, ws.forces, (ws.virial if stress else None)
        E, F, V, st = to_host(ws.energy, ws.forces, ws.virial if stress else None,
                              refresh.status[:1])
        if int(st[0]) != TopologyRefresh.OK:
            self._refresh_key = self._full_step = None
            return None
        return float(E[0]), F, V

    def _evaluate(self, pos, Z, cell, pbc, forces=True, stress=False, device_out=False,
                  charge=0.0, spin=0.0, defer_status=False):
        skey = self._system_key(Z, cell, pbc, forces, stress, charge, spin)
        self._pending_status = None
        if self.trace:
            fast = self._refresh_step(pos, skey, forces, stress, device_out, defer_status)
            if fast is not None:
                return fast
        g = build_graph(pos, Z, self.cfg["cutoff"], cell, pbc, max_neighbors=self.max_nbrs,
                        device=self.device)
        if g.E == 0:
            raise ValueError("no edges within cutoff — system too sparse for this model")
        if self._ws is None or not self._ws.fits(g):
            self._ws = self._step = self._full_step = None   # free the old buffers first
            self._ws = self.engine.workspace(g)
        else:
            self._ws.rebind(g)                  # same sizes: reuse the buffers
        ws = self._ws
        upload_positions(ws, pos)
        self.engine.set_condition(ws, charge, spin)       # OrbMol checkpoints only
        key = (g.N, g.E, bool(forces), bool(stress))
        if self.trace:
            if self._step is None or self._step_key != key:
                self._step = CapturedStep(self.engine, ws, forces=forces, virial=stress)
                self._step_key = key
            self._step()
        else:
            self.engine.run(ws, forces=forces, virial=stress)
        # a later traced call on this system may rebuild its list on the device in the graph
        self._refresh_key = skey if (self.trace and g.nsys == 1) else None
        if device_out:      # device tensors the next call overwrites
            return ws.energy, ws.forces, (ws.virial if stress else None)
        E, F, V = to_host(ws.energy, ws.forces, ws.virial if stress else None)
        return float(E[0]), F, V

    def calculate(self, atoms=None, properties=("energy", "forces"), system_changes=all_changes):
        super().calculate(atoms, properties, system_changes)
        pos = np.asarray(atoms.get_positions(), np.float32)
        Z = np.asarray(atoms.get_atomic_numbers(), np.int64)
        pbc = np.asarray(atoms.get_pbc())
        cell = np.asarray(atoms.get_cell(), np.float32) if pbc.any() else None
        want_stress = cell is not None and ("stress" in properties or bool(pbc.all()))
        charge = float(atoms.info.get("charge", 0.0))
        spin = float(atoms.info.get("spin", 0.0))
        if self.engine.direct:
            return self._calculate_direct(atoms, pos, Z, cell, pbc, properties, want_stress,
                                          charge, spin)
        # model pass and ZBL term on the device, then one read-back of all their results (and
        # of the neighbour-list refresh status when the traced step rebuilt the list)
        Ed, Fd, Vd = self._evaluate(pos, Z, cell, pbc if pbc.any() else None, True, want_stress,
                                    device_out=True, charge=charge, spin=spin,
                                    defer_status=True)
        zb = self._zbl_launch(self._ws, want_stress) if self.zbl else (None, None, None)
        status = self._pending_status
        E, F, V, Ez, Fz, Vz, st = to_host(Ed, Fd, Vd, *zb, status)
        if st is not None and int(st[0]) != 0:
            # the edge count changed: the step ran on the old topology; rebuild and redo
            self._refresh_key = self._full_step = None
            return self.calculate(atoms, properties, system_changes)
        E = float(E[0])
        n = len(Z)
        w = self._w
        E = energy_denormalize(E, Z, w)
        scale = conservative_scale(w, n)
        self.results["energy"] = self.results["free_energy"] = E
        self.results["energies"] = np.full(n, E / n)
        self.results["forces"] = (scale * F).numpy()
        S = conservative_stress(V.numpy(), n, atoms.get_cell(), w) if V is not None else None
        if self.zbl:
            Ez = float(Ez[0])
            self.results["energy"] = self.results["free_energy"] = E = E + Ez
            self.results["energies"] = np.full(n, E / n)
            self.results["forces"] = self.results["forces"] + Fz.numpy()
            if S is not None:
                S = S + voigt_6(Vz.numpy() / atoms_volume(atoms))
        if S is not None:
            self.results["stress"] = S

    def _device_energy_forces(self, pos, Z, cell, pbc, charge=0.0, spin=0.0):
        """Energy (float64 device scalar) and forces ([N, 3] float64 on the device) as
        ``calculate`` reports them -- normaliser and ZBL term included -- for the GPU-resident
        relaxation / MD loops; ``pos`` may be a device tensor. Direct checkpoints go through
        their heads on the host and are copied back."""
        n = len(Z)
        if self.engine.direct:
            E, F, _ = self._evaluate_direct(pos, Z, cell, pbc, False, charge, spin)
            w = self._w
            F = force_denormalize(F, w)
            E = energy_denormalize(E, Z, w)
            if self.zbl:
                Ez, Fz, _ = self._zbl(self._ws, False, scale=1.0)
                E, F = E + Ez, F + Fz
            return (torch.tensor(E, dtype=torch.float64, device=self.device),
                    F.to(self.device))
        Ed, Fd, _ = self._evaluate(pos, Z, cell, pbc, True, False, device_out=True, charge=charge,
                                   spin=spin)
        E, F = Ed[0].double(), Fd.double()
        w = self._w
        E = energy_denormalize(E, Z, w)
        F = F * conservative_scale(w, n)
        if self.zbl:
            zE, zF, _ = self._zbl_launch(self._ws, False)
            E, F = E + zE[0], F + zF.double()
        return E, F

    def close(self):
        """Release the device workspace and any captured step (tt_atom/ase_base.py:33)."""
        self._ws = None
        self._step = self._step_key = None
        self._full_step = self._refresh_key = None

    def evaluate_batch(self, systems, properties=("energy", "forces")):
        """Energies (and forces) of several systems (tt_atom/orb_calculator.py:217-327): the same
        result dict, ``energy`` [K] and ``forces`` (list of [N_k, 3]) or None. Orb bakes no
        per-composition routing, so compositions, charges and spins may mix. Evaluated one system
        per device pass through ``calculate`` (same normaliser and ZBL term), not as one
        disjoint-union pass."""
        from .calculator import _fields
        from .ase_compat import SimpleAtoms
        if len(systems) == 0:
            raise ValueError("empty batch")
        want_forces = "forces" in properties
        props = ("energy", "forces") if want_forces else ("energy",)
        energies, forces = [], []
        for s in systems:
            pos, Z, charge, spin, cell, pbc = _fields(s)
            a = SimpleAtoms(Z, pos, cell, pbc if pbc is not None else False,
                            info=dict(charge=charge, spin=spin))
            self.calculate(a, props)
            energies.append(float(self.results["energy"]))
            if want_forces:
                forces.append(np.asarray(self.results["forces"], dtype=np.float64).copy())
        return dict(energy=np.array(energies), forces=forces if want_forces else None)

    def _calculate_direct(self, atoms, pos, Z, cell, pbc, properties, want_stress, charge=0.0,
                          spin=0.0):
        """Direct checkpoints (tt_atom/orb_calculator.py:137-186): energy through the energy
        head's normaliser, forces and stress from their heads through their own normalisers,
        each plus the ZBL term summed over atoms."""
        if "stress" in properties and cell is not None and not self.engine.has_stress_head:
            raise ValueError("stress requested but this direct checkpoint carries no "
                             "stress_head weights.")
        want_stress = want_stress and self.engine.has_stress_head
        E, F, S = self._evaluate_direct(pos, Z, cell, pbc if pbc.any() else None, want_stress,
                                        charge, spin)
        n = len(Z)
        w = self._w

        E = energy_denormalize(E, Z, w)
        F = force_denormalize(F, w)
        if S is not None:
            S = stress_denormalize(S, w)
        if self.zbl:
            Ez, Fz, Vz = self._zbl(self._ws, S is not None, scale=1.0)
            E = E + Ez
            F = F + Fz
            if S is not None:
                S = S + torch.as_tensor(voigt_6(Vz.numpy() / atoms_volume(atoms)))
        self.results["energy"] = self.results["free_energy"] = E
        self.results["energies"] = np.full(n, E / n)
        self.results["forces"] = F.numpy()
        if S is not None:
            self.results["stress"] = S.numpy()
