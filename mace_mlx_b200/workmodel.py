"""Algorithmic work of each kernel of the step, per launch.

FLOPs count a multiply-add as 2 and include only input-gradient work in the
backward (no weight gradients, no recomputation).  Bytes are the compulsory
HBM traffic: every tensor the kernel must read or write once.  These figures
are the numerators of the roofline fractions ``bench.py`` reports.
"""

from __future__ import annotations

from .spec import ModelSpec

F32 = 4


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


def kernel_work(spec: ModelSpec, N: int, E: int) -> dict[tuple[str, int], dict]:
    """{(kernel name, layer): {"flops": F, "bytes": B}} for one evaluation."""
    out: dict[tuple[str, int], dict] = {}
    C = spec.C
    nb = spec.num_bessel
    nsh = (spec.max_ell + 1) ** 2
    out[("edge_fwd", -1)] = {"flops": E * (60 + 150 + 30 * nb), "bytes": E * (3 * 4 + 3 * F32 + 16 * F32 + nb * F32)}
    out[("edge_bwd", -1)] = {"flops": E * (60 + 400 + 40 * nb), "bytes": E * (16 * F32 + nb * F32 + 3 * F32 + 3 * F32)}
    out[("forces", -1)] = {"flops": E * 6, "bytes": E * (3 * F32 * 2 + 4 * 2) + N * 3 * F32}
    out[("embed", -1)] = {"flops": 0, "bytes": N * C * F32}
    out[("energy", -1)] = {"flops": N * spec.num_interactions, "bytes": N * (spec.num_interactions + 2) * F32}
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
        mlp_flops = 2 * E * sum(widths[j] * widths[j + 1] for j in range(len(widths) - 1))
        out[("mlp_fwd", t)] = {"flops": mlp_flops, "bytes": E * (nb + nh * H + W) * F32}
        out[("mlp_bwd", t)] = {"flops": mlp_flops, "bytes": E * (W + nh * H + 2 * nb) * F32}
        s_fwd = s_m = s_bwd = 0
        for ins in lay.conv.instrs:
            d1, d2, d3 = _d(ins.l1), _d(ins.l2), _d(ins.l3)
            s_fwd += 2 * (d1 * d3 + d3)
            s_m += 2 * d1 * d2 * d3
            s_bwd += 6 * d1 * d3 + 2 * d1 * d2 * d3 + 2 * d3 + 3 * d1
        out[("conv_fwd", t)] = {
            "flops": E * (C * s_fwd + s_m),
            "bytes": (E * (W + nsh + 2) + N * (in_dim + mid_dim)) * F32,
        }
        out[("conv_bwd", t)] = {
            "flops": E * (C * s_bwd + s_m),
            "bytes": (E * (2 * W + 2 * nsh + 2) + N * (in_dim * 2 + mid_dim)) * F32,
        }

        def lin(lspec, n_rows_per_node=None):
            fl = 0
            for ins in lspec.instrs:
                fl += 2 * N * ins.dim * ins.mul_in * ins.mul_out
            wb = sum(ins.mul_in * ins.mul_out for ins in lspec.instrs) * F32
            return {"flops": fl, "bytes": N * (lspec.irreps_in.dim + lspec.irreps_out.dim) * F32 + wb}

        out[("linear_up", t)] = lin(lay.linear_up)
        out[("linear_up_bwd", t)] = lin(lay.linear_up)
        out[("linear_msg", t)] = lin(lay.linear)
        out[("linear_msg_bwd", t)] = lin(lay.linear)
        out[("linear_prod", t)] = lin(lay.prod_linear)
        out[("linear_prod_bwd", t)] = lin(lay.prod_linear)
        sk = {"flops": sum(2 * N * i.dim * i.mul1 * i.mul_out for i in lay.skip.instrs),
              "bytes": N * (lay.skip.irreps_in1.dim + lay.skip.irreps_out.dim) * F32}
        out[("skip_fwd", t)] = sk
        out[("skip_bwd", t)] = sk
        # symmetric contraction as the polynomial of pack.sc_polynomial: per entry of
        # degree nu, nu multiplies + 1 add forward, 3*nu - 1 multiply-adds backward
        sc_f = sc_b = 0
        for o in lay.sc.outputs:
            for nu, n_e in _sc_entry_counts(o).items():
                sc_f += n_e * (nu + 1)
                sc_b += n_e * (3 * nu + 1)
        out[("sc_fwd", t)] = {"flops": N * C * sc_f, "bytes": N * (inter_dim + hid_dim) * F32}
        out[("sc_bwd", t)] = {"flops": N * C * sc_b, "bytes": N * (2 * inter_dim + hid_dim) * F32}
        ro = 2 * N * C * (16 if lay.readout_nonlinear else 1) * (2 if lay.readout_nonlinear else 1)
        out[("readout", t)] = {"flops": ro, "bytes": N * (hid_dim * 2) * F32}
    return out


def step_totals(spec: ModelSpec, N: int, E: int) -> dict:
    w = kernel_work(spec, N, E)
    return {"flops": sum(v["flops"] for v in w.values()), "bytes": sum(v["bytes"] for v in w.values())}
