"""Algorithmic work of each kernel of the step, per evaluation.

For every (kernel, layer) three figures:

* ``flops`` -- the arithmetic the kernel performs as written, a multiply-add
  counted as 2, input-gradient work only in the backward (no weight
  gradients) and no recomputation.  The conv kernels are counted in the form
  they compute: the forward forms ``M_k = CG_k . Y_e`` once per edge and then
  ``t = x . M_k``, ``acc += w t`` per channel; the backward contracts CG with
  the receiver's gradient once per receiver (the H tables) and then spends,
  per edge, path and channel, ``2 d1 d2`` (x.H) ``+ 2 d1 d2`` (H.Y, input
  gradient) ``+ 2 d1 + 4 d2`` (sender term, dw, dY).
* ``bytes`` -- the compulsory HBM traffic of the reference's data flow
  (node-feature tables read or written once, the edge list at 11 bytes per
  edge: sender, receiver, three int8 shifts, plus positions where the kernel's
  inputs are positions), i.e. what a fully fused step would still have to
  move.
* ``bytes_materialised`` -- per-edge intermediates this implementation keeps
  in HBM between kernels (radial-MLP outputs ``w`` and their gradient ``dw``,
  hidden activations, SH and radial-basis rows, the backward's per-edge
  sender terms); ``bytes + bytes_materialised`` is what the kernel reads and
  writes by design, which ncu's DRAM counters are compared with.

``bench.py`` divides these by event-timed kernel durations for the roofline.
"""

from __future__ import annotations

from .spec import ModelSpec

F32 = 4
EDGE_LIST = 11  # bytes per directed edge: int32 sender + int32 receiver + 3 x int8 shift


def _d(l: int) -> int:
    return 2 * l + 1


def _sc_entry_counts(out) -> dict[int, int]:
    """Entries per degree nu of the symmetrised polynomial of one SC output."""
    import numpy as np

    counts = {}
    for nu, U in enumerate(out.U, start=1):
        u = U[None] if out.ir_out.l == 0 else U
        nz = np.argwhere(np.abs(u) > 1e-12)
        keys = {(r[0],) + tuple(sorted(r[1:1 + nu])) for r in nz}
        counts[nu] = len(keys)
    return counts


def _w(flops, bytes_, mat=0):
    return {"flops": int(flops), "bytes": int(bytes_), "bytes_materialised": int(mat)}


def kernel_work(spec: ModelSpec, N: int, E: int) -> dict[tuple[str, int], dict]:
    """{(kernel name, layer): {"flops", "bytes", "bytes_materialised"}} for one evaluation."""
    out: dict[tuple[str, int], dict] = {}
    C = spec.C
    nb = spec.num_bessel
    nsh = (spec.max_ell + 1) ** 2
    # edge front end: positions + edge list in; SH rows and radial basis out
    out[("edge_fwd", -1)] = _w(E * (60 + 150 + 30 * nb), N * 3 * F32 + E * EDGE_LIST, E * (nsh + nb + 3) * F32)
    out[("edge_bwd", -1)] = _w(E * (60 + 400 + 40 * nb), E * EDGE_LIST, E * (2 * nsh + 2 * nb + 3 + 3) * F32)
    out[("forces", -1)] = _w(E * 6, E * (EDGE_LIST + 4) + N * 3 * F32, E * 3 * F32)
    out[("embed", -1)] = _w(0, N * C * F32)
    out[("energy", -1)] = _w(N * spec.num_interactions, N * (spec.num_interactions + 2) * F32)
    if spec.density or spec.zbl:
        out[("node_sums", -1)] = _w(E * (2 * nb + 2) * sum(lay.density for lay in spec.layers)
                                    + (E * 60 if spec.zbl else 0), E * EDGE_LIST + N * 4 * F32,
                                    E * (nb + 3) * F32)
    for lay in spec.layers:
        t = lay.index
        W = lay.conv.weight_numel
        widths = lay.mlp_widths
        H = widths[1]
        nh = len(widths) - 2
        in_dim = lay.irreps_in.dim
        mid_dim = lay.conv.irreps_mid.dim
        inter_dim = spec.interaction_irreps.dim
        hid_dim = lay.hidden.dim
        n_in_ch = sum(m.ir.dim for m in lay.irreps_in)
        mlp_flops = 2 * E * sum(widths[j] * widths[j + 1] for j in range(len(widths) - 1))
        # the radial MLP reads the basis rows and writes the weights (both per-edge intermediates)
        out[("mlp_fwd", t)] = _w(mlp_flops, 0, E * (nb + nh * H + W) * F32)
        out[("mlp_bwd", t)] = _w(mlp_flops, 0, E * (W + nh * H + 2 * nb) * F32)
        f_edge = f_chan = b_chan = b_recv = 0
        need_dup = t > 0  # layer 0's input is the species embedding: no input gradient
        for ins in lay.conv.instrs:
            d1, d2, d3 = _d(ins.l1), _d(ins.l2), _d(ins.l3)
            f_edge += 2 * d1 * d2 * d3              # M_k = CG . Y, once per edge
            f_chan += 2 * (d1 * d3 + d3)            # t = x . M, acc += w t
            b_recv += 2 * d1 * d2 * d3              # H_k = CG . dA, once per receiver and channel
            b_chan += 2 * d1 * d2 + 4 * d2          # x . H, dw, dY
            if need_dup:
                b_chan += 2 * d1 * d2 + 2 * d1      # H . Y and the sender term
        nodes_fwd = N * (in_dim + mid_dim) * F32
        out[("conv_fwd", t)] = _w(E * (f_edge + C * f_chan), nodes_fwd + E * EDGE_LIST, E * (W + nsh) * F32)
        nodes_bwd = N * (in_dim + mid_dim + (in_dim if need_dup else 0)) * F32
        out[("conv_bwd", t)] = _w(E * C * b_chan + N * C * b_recv, nodes_bwd + E * EDGE_LIST,
                                  E * (2 * W + 2 * nsh + (n_in_ch * C if need_dup else 0)) * F32)
        if need_dup:
            out[("dup_gather", t)] = _w(E * n_in_ch * C, N * in_dim * F32 + E * 4, E * n_in_ch * C * F32)

        def lin(lspec):
            fl = 0
            for ins in lspec.instrs:
                fl += 2 * N * ins.dim * ins.mul_in * ins.mul_out
            wb = sum(ins.mul_in * ins.mul_out for ins in lspec.instrs) * F32
            return _w(fl, N * (lspec.irreps_in.dim + lspec.irreps_out.dim) * F32 + wb)

        sk = _w(sum(2 * N * i.dim * i.mul1 * i.mul_out for i in lay.skip.instrs),
                N * (lay.skip.irreps_in1.dim + lay.skip.irreps_out.dim) * F32)
        up = lin(lay.linear_up)
        if lay.residual:  # linear_up and the residual skip share one launch
            out[("linear_up+skip", t)] = _w(up["flops"] + sk["flops"], up["bytes"] + N * hid_dim * F32)
        else:
            out[("linear_up+skip", t)] = up
            out[("skip_fwd", t)] = sk
        if t > 0:
            out[("linear_up_bwd", t)] = lin(lay.linear_up)
        if t > 0 or not lay.residual:
            out[("skip_bwd", t)] = sk
        out[("linear_msg", t)] = lin(lay.linear)
        out[("linear_msg_bwd", t)] = lin(lay.linear)
        out[("linear_prod", t)] = lin(lay.prod_linear)
        out[("linear_prod_bwd", t)] = lin(lay.prod_linear)
        if lay.density:
            out[("density_scale", t)] = _w(N * inter_dim, 2 * N * inter_dim * F32)
            out[("density_bwd", t)] = _w(3 * N * inter_dim, 3 * N * inter_dim * F32)
        # symmetric contraction as the polynomial of pack.sc_polynomial: per entry of
        # degree nu, nu multiplies + 1 add forward, 3*nu - 1 multiply-adds backward
        sc_f = sc_b = 0
        for o in lay.sc.outputs:
            for nu, n_e in _sc_entry_counts(o).items():
                sc_f += n_e * (nu + 1)
                sc_b += n_e * (3 * nu + 1)
        out[("sc_fwd", t)] = _w(N * C * sc_f, N * (inter_dim + hid_dim) * F32)
        out[("sc_bwd", t)] = _w(N * C * sc_b, N * (2 * inter_dim + hid_dim) * F32)
        ro = 2 * N * C * (16 if lay.readout_nonlinear else 1) * (2 if lay.readout_nonlinear else 1)
        out[("readout", t)] = _w(ro, N * (hid_dim * 2) * F32)
    return out


def step_totals(spec: ModelSpec, N: int, E: int) -> dict:
    w = kernel_work(spec, N, E)
    return {k: sum(v[k] for v in w.values()) for k in ("flops", "bytes", "bytes_materialised")}
